"""``torch.ops.flashdec.*`` (flashdec_b200.ops) on the CPU: the operators are
registered and their fake implementations give torch.compile the output's
shape and dtype without running anything."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")


def test_ops_registered_with_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import flashdec_b200.ops  # noqa: F401

    assert hasattr(torch.ops.flashdec, "decode") and hasattr(torch.ops.flashdec, "decode_into")
    with FakeTensorMode():
        q = torch.empty(8, 16, 128, dtype=torch.bfloat16)
        k = torch.empty(64, 2, 32, 128, dtype=torch.bfloat16)
        bt = torch.empty(8, 8, dtype=torch.int32)
        sl = torch.empty(8, dtype=torch.int32)
        out = torch.ops.flashdec.decode(q, k, k, bt, sl)
        assert out.shape == q.shape and out.dtype == q.dtype
        assert torch.ops.flashdec.decode_into(q, k, k, bt, sl, torch.empty_like(q)) is None
