"""K + V pair boxes of the one-wave kernel (one TMA copy moves a page's K and
V) against the per-plane boxes (FLASHDEC_B200_KV_PAIR=0), bit for bit, in
child processes:

* 32-token pages with the planes in two allocations (the c2 layout);
* 16-token pages with the planes in two allocations (HND);
* vLLM's cache, [block, 2, 16, kv_head, dim] with K and V interleaved per
  block, through the vLLM launcher with the fused current-token append
  (outputs and the cache bytes after the append).

Both paths read the same bytes into the same positions of the tile, so the
arithmetic and its order are the same: any layout mistake in the pair path
shows as a bit difference."""

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
from flashdec_b200.kernels.paged_decode import _vllm_paged_decode_attention_into
from tests.golden.cases import _normal
rng = np.random.default_rng(11)
out = {{}}

def t(a):
    return torch.from_numpy(a).to(torch.bfloat16).cuda()

for name, (b, ctx, bs) in {{"bs32": (8, 2048, 32), "bs16": (4, 700, 16)}}.items():
    nblk = -(-ctx // bs)
    pool = 2 * b * nblk
    q = t(_normal(rng, (b, 16, 128), "bfloat16"))
    k = t(_normal(rng, (pool, 2, bs, 128), "bfloat16"))
    v = t(_normal(rng, (pool, 2, bs, 128), "bfloat16"))
    bt = torch.from_numpy(rng.permutation(pool)[: b * nblk].reshape(b, nblk).astype(np.int32)).cuda()
    sl = torch.full((b,), ctx, dtype=torch.int32).cuda()
    o = torch.empty_like(q)
    for _ in range(3):
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, o)
    torch.cuda.synchronize()
    out[name] = o.view(torch.int16).cpu().numpy()

# vLLM: B8 ragged lengths, 16-token NHD pages, fused append of the current token
b, bs, hkv = 8, 16, 2
lens = [2048, 1, 17, 640, 1999, 33, 1024, 16]
nblk = [-(-n // bs) for n in lens]
pool = sum(nblk) + 8
kv = t(_normal(rng, (pool, 2, bs, hkv, 128), "bfloat16"))
perm = rng.permutation(pool)
bt = np.full((b, max(nblk)), 0, np.int32)
at = 0
for i, n in enumerate(nblk):
    bt[i, :n] = perm[at:at + n]
    at += n
btd = torch.from_numpy(bt).cuda()
sl = torch.tensor(lens, dtype=torch.int32).cuda()
pos = torch.tensor(lens, dtype=torch.int64) - 1
slots = (torch.from_numpy(bt).long().gather(1, (pos // bs)[:, None])[:, 0] * bs + pos % bs).cuda()
q = t(_normal(rng, (b, 16, 128), "bfloat16"))
ak = t(_normal(rng, (b, hkv, 128), "bfloat16"))
av = t(_normal(rng, (b, hkv, 128), "bfloat16"))
o = torch.empty_like(q)
acc = torch.empty((b, 16, 16, 128), dtype=torch.float32, device="cuda")
mx = torch.empty((b, 16, 16), dtype=torch.float32, device="cuda")
sm = torch.empty_like(mx)
_vllm_paged_decode_attention_into(q, ak, av, kv, btd, sl, o, slots, acc, mx, sm,
                                  num_reqs=b, num_q_heads=16, num_kv_heads=hkv, head_dim=128,
                                  block_size=bs, sm_scale=128 ** -0.5, num_splits=0)
torch.cuda.synchronize()
assert flashdec_b200.device_status() == 0
out["vllm_out"] = o.view(torch.int16).cpu().numpy()
out["vllm_cache"] = kv.view(torch.int16).cpu().numpy()
np.savez({path!r}, **out)
"""


def _run(tmp_path, pair):
    path = str(tmp_path / f"out_{pair}.npz")
    env = dict(os.environ, FLASHDEC_B200_KV_PAIR=str(pair))
    res = subprocess.run([sys.executable, "-c", _CHILD.format(root=str(ROOT), path=path)],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    return dict(np.load(path))


def test_pair_boxes_match_plane_boxes_bit_for_bit(tmp_path):
    pair = _run(tmp_path, 1)
    planes = _run(tmp_path, 0)
    assert pair.keys() == planes.keys()
    for name in pair:
        assert np.array_equal(pair[name], planes[name]), name
