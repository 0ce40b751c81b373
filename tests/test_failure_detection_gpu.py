"""Failure detection without a GPU fault.

Every wait in the library's kernels is bounded: when it runs out, the kernel
records FD_STATUS_WAIT_TIMEOUT in the device status word and unwinds instead
of hanging.  ``fd_selftest_wait_timeout`` drives that exact wait routine
against a barrier nothing arrives on, with a short limit; the host then reads
the status word and the context must still run a correct decode."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.paged_attention import paged_decode_attention_ref  # noqa: E402
from tests.golden.cases import make_attn_case  # noqa: E402
from tests.helpers import assert_attention_close, to_dev, to_np  # noqa: E402

pytestmark = pytest.mark.gpu


def _lib():
    from flashdec_b200 import _lib

    return _lib, _lib.load_library()


def test_bounded_wait_timeout_sets_status_and_context_survives():
    import flashdec_b200

    _l, lib = _lib()
    flashdec_b200.device_status(clear=True)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _l.check(lib.fd_selftest_wait_timeout(50_000_000, ctypes.c_void_p(stream.cuda_stream)),
             "fd_selftest_wait_timeout")
    e1.record(stream)
    torch.cuda.synchronize()
    waited_ms = e0.elapsed_time(e1)
    assert 50.0 <= waited_ms < 2000.0, waited_ms
    assert flashdec_b200.device_status(clear=True) == _l.FD_STATUS_WAIT_TIMEOUT
    assert flashdec_b200.device_status() == 0

    # the context is intact: a decode right after is correct and clean
    c = make_attn_case("split_257_193")
    out = flashdec_b200.decode(to_dev(c["q"], c["dtype"]), to_dev(c["k_cache"], c["dtype"]),
                               to_dev(c["v_cache"], c["dtype"]), to_dev(c["block_tables"]),
                               to_dev(c["seq_lens"]))
    want = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"])
    assert_attention_close(to_np(out), want)
    assert flashdec_b200.device_status() == 0


def test_selftest_rejects_unbounded_limits():
    _l, lib = _lib()
    assert lib.fd_selftest_wait_timeout(0, None) == _l.FD_ERR_INVALID_ARGUMENT
    assert lib.fd_selftest_wait_timeout(10_000_000_000, None) == _l.FD_ERR_INVALID_ARGUMENT


def test_decode_replays_inside_a_cuda_graph():
    """The checked API is capturable once the workspace exists: replays of
    the captured launch match eager results and the oracle, including after
    the inputs change in place."""
    import flashdec_b200

    c = make_attn_case("c2_ctx1024")
    q = to_dev(c["q"], c["dtype"])
    k, v = to_dev(c["k_cache"], c["dtype"]), to_dev(c["v_cache"], c["dtype"])
    bt, sl = to_dev(c["block_tables"]), to_dev(c["seq_lens"])
    out = torch.empty_like(q)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)  # sizes the workspace
    stream.synchronize()
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    want = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"])
    assert_attention_close(to_np(out), want)
    # new query values in the same buffer: the replay reads them
    rng = np.random.default_rng(9)
    from tests.golden.cases import _normal

    q2 = _normal(rng, c["q"].shape, c["dtype"])
    q.copy_(to_dev(q2, c["dtype"]))
    graph.replay()
    torch.cuda.synchronize()
    want2 = paged_decode_attention_ref(q2, c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"])
    assert_attention_close(to_np(out), want2)
    assert flashdec_b200.device_status() == 0
