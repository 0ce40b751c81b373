"""The C++ host path module (flashdec_b200._hostpath) on the CPU: it loads
against this build's C ABI, never takes CPU tensors (a miss sends the call to
the Python path, which raises the reference's errors), splits packed engine
metadata into the right typed views, and rejects a layer's q/k/v with the
engine's messages before any launch."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def hp():
    from flashdec_b200 import _lib

    try:
        return _lib.load_hostpath()
    except RuntimeError as exc:  # library not built in this checkout
        pytest.skip(str(exc))


def test_module_matches_the_c_abi(hp):
    from flashdec_b200 import _lib

    assert hp.ARGS_BYTES == ctypes.sizeof(_lib.PagedDecodeArgs)
    assert hp.MISS == 1


def test_cpu_tensors_are_a_miss(hp):
    from flashdec_b200 import _lib

    q = torch.zeros((2, 4, 128), dtype=torch.bfloat16)
    assert hp.decode_into(q, q, q, q, q, q) == hp.MISS
    args = _lib.PagedDecodeArgs()
    assert hp.register_decode(q, q, q, q, q, q, ctypes.addressof(args)) is False


def test_unpack_meta_views(hp):
    from flashdec_b200.cache import _unpack_meta

    n = 5
    rng = np.random.default_rng(0)
    packed = np.empty(4 * n * 8 + n * 4, np.uint8)
    i64 = packed[:4 * n * 8].view(np.int64)
    i64[:] = rng.integers(-5, 1 << 40, size=4 * n)
    packed[4 * n * 8:].view(np.int32)[:] = rng.integers(0, 1 << 20, size=n)
    buf = torch.from_numpy(packed)
    got = hp.unpack_meta(buf, n)
    want = _unpack_meta(buf, n)
    assert len(got) == 5
    for g, w in zip(got, want):
        assert g.dtype == w.dtype and g.shape == w.shape and torch.equal(g, w)
        assert g.data_ptr() == w.data_ptr()  # views of the buffer, no copy


def test_layer_run_rejects_shapes_with_the_engine_messages(hp):
    from flashdec_b200 import _lib

    a = _lib.PagedDecodeArgs()
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim = 2, 8, 2, 128
    addr = ctypes.addressof(a)
    q = torch.zeros((2, 8, 128), dtype=torch.bfloat16)
    k = torch.zeros((2, 2, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="q must be a contiguous"):
        hp.layer_run(addr, 0, q.transpose(0, 1).contiguous().transpose(0, 1), k, k, 0, 0)
    with pytest.raises(ValueError, match="q must be a contiguous"):
        hp.layer_run(addr, 0, q[:1], k, k, 0, 0)
    with pytest.raises(ValueError, match="k and v must be contiguous"):
        hp.layer_run(addr, 0, q, k[:, :1], k, 0, 0)
    with pytest.raises(ValueError, match="current CUDA device"):
        hp.layer_run(addr, 0, q, k, k, 0, 0)


def test_copy_async_rejects_misuse_before_any_cuda_call(hp):
    import flashdec_b200

    assert flashdec_b200.copy_async is hp.copy_async
    a = torch.zeros(8)
    with pytest.raises(ValueError, match="one of dst and src must be a CUDA tensor"):
        hp.copy_async(a, torch.ones(8))
    with pytest.raises(ValueError, match="one of dst and src must be a CUDA tensor"):
        hp.copy_async(a[::2], torch.ones(4))
    with pytest.raises(TypeError):
        hp.copy_async(a, None)
