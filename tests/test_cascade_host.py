"""Host-side checks of the cascade (shared-prefix) group description; the
kernels are exercised in tests/test_cascade_gpu.py."""

from __future__ import annotations

import ctypes

import pytest

torch = pytest.importorskip("torch")


def test_group_description_is_checked():
    from flashdec_b200 import _native

    with pytest.raises(ValueError, match="multiple of 32"):
        _native.CascadeGroups([[0, 1]], [3], 2, 16, "cpu")
    with pytest.raises(ValueError, match="distinct"):
        _native.CascadeGroups([[0, 1], [1]], [2, 2], 2, 32, "cpu")
    with pytest.raises(ValueError, match="distinct"):
        _native.CascadeGroups([[0, 5]], [2], 2, 32, "cpu")
    with pytest.raises(ValueError, match="one page count"):
        _native.CascadeGroups([], [], 2, 32, "cpu")


def test_group_description_layout():
    from flashdec_b200 import _lib, _native

    g = _native.CascadeGroups([[3, 1], [0]], [4, 2], 5, 16, "cpu")
    assert list(g.host_start) == [0, 2, 3]
    assert list(g.host_members) == [3, 1, 0]
    assert list(g.host_pages) == [4, 2]
    assert g.seq_pages.tolist() == [2, 4, 0, 4, 0]
    a = g.args
    assert a.struct_size == ctypes.sizeof(_lib.CascadeArgs)
    assert a.num_groups == 2
    assert a.group_start == ctypes.addressof(g.host_start)
    assert a.seq_prefix_pages == g.seq_pages.data_ptr()


def test_cascade_host_checks_answer_without_a_gpu():
    """The C-ABI checks the (host) group description before touching a GPU."""
    from flashdec_b200 import _lib

    lib = _lib.load_library()
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a)
    a.dtype, a.head_dim, a.block_size = _lib.FD_DTYPE_BF16, 128, 16
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq = 3, 8, 1, 8, 8
    a.q = a.out = a.k_cache = a.v_cache = a.block_tables = a.seq_lens = 1
    start = (ctypes.c_int32 * 2)(0, 2)
    members = (ctypes.c_int32 * 2)(0, 1)
    pages = (ctypes.c_int32 * 1)(2)
    c = _lib.CascadeArgs()
    c.struct_size = ctypes.sizeof(c)
    c.num_groups = 1
    c.group_start, c.group_members = ctypes.addressof(start), ctypes.addressof(members)
    c.group_pages, c.seq_prefix_pages = ctypes.addressof(pages), 1
    bad = _lib.FD_ERR_INVALID_ARGUMENT
    pages[0] = 3  # 48 tokens: not whole 32-token tiles
    assert lib.fd_cascade_decode(ctypes.byref(a), ctypes.byref(c), None) == bad
    pages[0] = 2
    members[1] = 3  # not a row of the batch
    assert lib.fd_cascade_decode(ctypes.byref(a), ctypes.byref(c), None) == bad
    members[1] = 1
    start[1] = 0  # empty group
    assert lib.fd_cascade_decode(ctypes.byref(a), ctypes.byref(c), None) == bad
