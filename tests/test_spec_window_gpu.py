"""The one-wave small-batch kernel may issue its first tiles from a block
table read before griddepcontrol.wait (while the previous kernel of the
stream may still be writing it) and checks them against the real table once
that arrives, loading any wrong tile again.  With
FLASHDEC_B200_TEST_SPEC_SKEW set, every speculatively read block id is
shifted, so every speculative tile is wrong and must be re-loaded: the
results must be the same bits as without the skew (the path the oracle
parity tests check)."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

_CHILD = r"""
import sys
sys.path.insert(0, {root!r})
import numpy as np, torch
import flashdec_b200
from tests.golden.cases import _normal
rng = np.random.default_rng(5)
out = {{}}
for name, (b, ctx, bs, d) in {{"c2": (8, 2048, 32, 128), "bs16": (4, 700, 16, 128),
                               "d64": (6, 333, 8, 64)}}.items():
    nblk = -(-ctx // bs)
    pool = 2 * b * nblk
    q = torch.from_numpy(_normal(rng, (b, 16, d), "bfloat16")).to(torch.bfloat16).cuda()
    k = torch.from_numpy(_normal(rng, (pool, 2, bs, d), "bfloat16")).to(torch.bfloat16).cuda()
    v = torch.from_numpy(_normal(rng, (pool, 2, bs, d), "bfloat16")).to(torch.bfloat16).cuda()
    bt = torch.from_numpy(rng.permutation(pool)[: b * nblk].reshape(b, nblk).astype(np.int32)).cuda()
    sl = torch.full((b,), ctx, dtype=torch.int32).cuda()
    o = torch.empty_like(q)
    for _ in range(3):  # back-to-back calls: the later ones run their speculative path
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, o)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status() == 0
    out[name] = o.view(torch.int16).cpu().numpy()
np.savez({path!r}, **out)
"""


def _run(tmp_path, skew):
    path = str(tmp_path / f"out_{skew}.npz")
    env = dict(os.environ)
    env.pop("FLASHDEC_B200_TEST_SPEC_SKEW", None)
    if skew:
        env["FLASHDEC_B200_TEST_SPEC_SKEW"] = str(skew)
    res = subprocess.run([sys.executable, "-c", _CHILD.format(root=str(ROOT), path=path)],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    return dict(np.load(path))


def test_wrong_speculative_pages_are_loaded_again(tmp_path):
    plain = _run(tmp_path, 0)
    skewed = _run(tmp_path, 7)
    assert plain.keys() == skewed.keys()
    for name in plain:
        assert np.array_equal(plain[name], skewed[name]), name
