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
    data = g.data.tolist()
    # group_start | members | pages | per-sequence prefix pages
    assert data == [0, 2, 3, 3, 1, 0, 4, 2, 2, 4, 0, 4, 0]
    a = g.args
    assert a.struct_size == ctypes.sizeof(_lib.CascadeArgs)
    assert a.num_groups == 2 and a.max_group_members == 2 and a.max_prefix_tiles == 2
    base = g.data.data_ptr()
    assert (a.group_start, a.group_members, a.group_pages, a.seq_prefix_pages) == (
        base, base + 12, base + 24, base + 32)
