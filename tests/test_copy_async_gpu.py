"""flashdec_b200.copy_async on the GPU: pinned host -> device, device ->
pinned host and device -> device copies of the bytes as stored (any dtype
pair of equal size), in order with the kernels of the current stream, and
ValueErrors for mismatched sizes, non-contiguous tensors, overlapping device
ranges and a CUDA tensor off the current device."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_round_trip_keeps_the_bytes():
    import flashdec_b200

    g = torch.Generator().manual_seed(3)
    host = torch.randn((8, 16, 128), generator=g).to(torch.bfloat16).pin_memory()
    dev = torch.empty_like(host, device="cuda")
    dev2 = torch.empty((8 * 16 * 128,), dtype=torch.int16, device="cuda")  # same bytes
    back = torch.zeros_like(host).pin_memory()
    flashdec_b200.copy_async(dev, host)
    flashdec_b200.copy_async(dev2, dev)
    flashdec_b200.copy_async(back, dev2)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(back, host)
    assert torch.equal(dev2.view(torch.bfloat16).view(host.shape).cpu(), host)


def test_copies_follow_the_current_stream():
    """A download issued after a decode on a side stream sees that decode's
    output; an upload issued after it does not disturb it."""
    import flashdec_b200

    g = torch.Generator(device="cuda").manual_seed(5)
    b, hq, hkv, d, bs, nblk = 4, 16, 2, 128, 32, 16
    k = torch.randn((b * nblk, hkv, bs, d), device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn_like(k)
    bt = torch.randperm(b * nblk, device="cuda", generator=g).reshape(b, nblk).to(torch.int32)
    sl = torch.full((b,), nblk * bs, device="cuda", dtype=torch.int32)
    q_host = [torch.randn((b, hq, d), dtype=torch.float32).to(torch.bfloat16).pin_memory()
              for _ in range(3)]
    want = [flashdec_b200.decode(x.cuda(), k, v, bt, sl).cpu() for x in q_host]
    side = torch.cuda.Stream()
    q_dev = torch.empty((b, hq, d), device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q_dev)
    got = [torch.empty((b, hq, d), dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        torch.cuda._sleep(1_000_000)  # the host runs ahead of the stream
        for i in range(3):
            flashdec_b200.copy_async(q_dev, q_host[i])
            flashdec_b200.paged_decode_attention_into(q_dev, k, v, bt, sl, out)
            flashdec_b200.copy_async(got[i], out)
    side.synchronize()
    assert flashdec_b200.device_status() == 0
    for i in range(3):
        assert torch.equal(got[i], want[i]), i


def test_misuse_raises_value_error():
    import flashdec_b200

    dev = torch.zeros(8, device="cuda")
    with pytest.raises(ValueError, match="same number of bytes"):
        flashdec_b200.copy_async(dev, torch.zeros(9))
    with pytest.raises(ValueError, match="contiguous"):
        flashdec_b200.copy_async(dev, torch.zeros(16)[::2])
    if torch.cuda.device_count() > 1:
        with pytest.raises(ValueError, match="current CUDA device"):
            flashdec_b200.copy_async(torch.zeros(8, device="cuda:1"), torch.zeros(8))
    buf = torch.zeros(16, device="cuda")
    with pytest.raises(ValueError, match="overlap"):
        flashdec_b200.copy_async(buf[4:12], buf[:8])
    flashdec_b200.copy_async(buf[8:], buf[:8])  # adjacent ranges are fine
    flashdec_b200.copy_async(torch.empty(0, device="cuda"), torch.empty(0))  # nothing to copy
