"""BASELINE config 4 at its real size on the GPU: 64 requests of the
Llama-3-8B attention shape (32 q / 8 KV heads, head_dim 128, 16-token pages,
bf16) with log-uniform lengths in [512, 131072] (seed 4, about 1.5 M tokens
and 6 GB of K/V), decoded through the public ``paged_decode_attention_into``
(the length-balanced stream-K plan) and through the C-ABI launch with
``max_ctas`` 37 and 148 (other cuts of the same batch).  The longest request
and three others are checked against the numpy oracle restating
flashdec/paged_reference.py:19-125; every plan must also agree with the
others on every request within the attention tolerance."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.paged_attention import paged_decode_attention_ref  # noqa: E402
from tests.golden.cases import c4_lengths  # noqa: E402
from tests.helpers import assert_attention_close, to_np  # noqa: E402

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 32, 8, 128, 16


@pytest.fixture(scope="module")
def c4():
    lens = c4_lengths()
    nblk = [-(-n // BS) for n in lens]
    total = sum(nblk)
    g = torch.Generator(device="cuda").manual_seed(4)
    k = torch.randn((total + 1, HKV, BS, D), device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn((total + 1, HKV, BS, D), device="cuda", dtype=torch.bfloat16, generator=g)
    perm = torch.randperm(total + 1, device="cuda", generator=g).to(torch.int32)
    bt = torch.full((len(lens), max(nblk)), -1, device="cuda", dtype=torch.int32)
    at = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[at:at + n]
        at += n
    sl = torch.tensor(lens, device="cuda", dtype=torch.int32)
    q = torch.randn((len(lens), HQ, D), device="cuda", dtype=torch.bfloat16, generator=g)
    return dict(lens=lens, nblk=nblk, k=k, v=v, bt=bt, sl=sl, q=q)


def _outputs(c4):
    import flashdec_b200
    from flashdec_b200 import _native

    outs = {}
    out = torch.empty_like(c4["q"])
    flashdec_b200.paged_decode_attention_into(c4["q"], c4["k"], c4["v"], c4["bt"], c4["sl"], out)
    outs["auto"] = out
    for ctas in (37, 148):
        out = torch.empty_like(c4["q"])
        _native.paged_decode(c4["q"], c4["k"], c4["v"], c4["bt"], c4["sl"], out,
                             sm_scale=D ** -0.5, block_size=BS, num_seqs=len(c4["lens"]),
                             num_splits=0, max_ctas=ctas)
        outs[f"max_ctas={ctas}"] = out
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    return outs


def _oracle_row(c4, i):
    """Oracle output of request i, from its own pages copied to the host."""
    n, nb = c4["lens"][i], c4["nblk"][i]
    blocks = c4["bt"][i, :nb].long()
    kc = c4["k"].index_select(0, blocks).float().cpu().numpy()
    vc = c4["v"].index_select(0, blocks).float().cpu().numpy()
    q = c4["q"][i:i + 1].float().cpu().numpy()
    bt = np.arange(nb, dtype=np.int32)[None]
    return paged_decode_attention_ref(q, kc, vc, bt, np.asarray([n], np.int32),
                                      sm_scale=D ** -0.5)


def test_c4_full_batch_matches_oracle(c4):
    outs = _outputs(c4)
    lens = np.asarray(c4["lens"])
    order = np.argsort(lens)
    picks = [int(order[-1]), int(order[0]), int(order[len(order) // 2]),
             int(order[(3 * len(order)) // 4])]
    for i in picks:
        want = _oracle_row(c4, i)
        for name, out in outs.items():
            try:
                assert_attention_close(to_np(out[i:i + 1]), want)
            except AssertionError as e:
                raise AssertionError(f"request {i} (length {lens[i]}), plan {name}: {e}") from e
    # every plan agrees with the default one on every request
    ref = to_np(outs["auto"])
    for name, out in outs.items():
        assert_attention_close(to_np(out), ref, max_abs=2e-2, mean_abs=2e-3)
