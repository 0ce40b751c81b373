"""The C-ABI boundary on the CPU: the library loads, exports every entry point
``include/flashdec_b200.h`` declares, its structs have the same layout as
the ctypes mirror, and host-side argument checks answer without a GPU.
No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from flashdec_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "flashdec_b200.h"

_STRUCTS = {
    "fd_paged_decode_args": _lib.PagedDecodeArgs,
    "fd_split_kv_reduce_args": _lib.SplitReduceArgs,
    "fd_rope_kv_append_args": _lib.RopeKVAppendArgs,
    "fd_cascade_args": _lib.CascadeArgs,
}


def declared_functions(text: str):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(fd_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.library_path().exists():
        pytest.fail("libflashdec_b200.so is not built (python -m flashdec_b200.build)")
    return _lib.load_library()


def test_header_declarations_match_the_binding_list():
    assert declared_functions(HEADER.read_text()) == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions(HEADER.read_text()):
        assert hasattr(lib, name), name
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_lib.library_path())],
                             capture_output=True, text=True, check=True).stdout
        exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
        for name in declared_functions(HEADER.read_text()):
            assert name in exported, name


def _c_layout(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "flashdec_b200.h"',
             "int main(void) {"]
    for cname, cls in _STRUCTS.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c99", "-I", str(HEADER.parent), str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    layout = {}
    for line in out.splitlines():
        s, f, v = line.split()
        layout[(s, f)] = int(v)
    return layout


def test_ctypes_structs_match_the_c_layout(tmp_path):
    layout = _c_layout(tmp_path)
    for cname, cls in _STRUCTS.items():
        assert layout[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert layout[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def test_version_and_error_strings(lib):
    assert lib.fd_version() == 1
    assert lib.fd_error_string(_lib.FD_OK) == b"ok"
    for code in (_lib.FD_ERR_INVALID_ARGUMENT, _lib.FD_ERR_UNSUPPORTED, _lib.FD_ERR_WORKSPACE,
                 _lib.FD_ERR_ALIGNMENT):
        msg = lib.fd_error_string(code)
        assert msg and msg != b"unknown error"
    assert lib.fd_error_string(12345) == b"unknown error"


def test_host_argument_checks_answer_without_a_gpu(lib):
    assert lib.fd_paged_decode(None, None) == _lib.FD_ERR_INVALID_ARGUMENT
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a) - 8  # stale struct version
    assert lib.fd_paged_decode(ctypes.byref(a), None) == _lib.FD_ERR_INVALID_ARGUMENT
    a.struct_size = ctypes.sizeof(a)
    a.dtype = _lib.FD_DTYPE_F32
    assert lib.fd_paged_decode(ctypes.byref(a), None) == _lib.FD_ERR_UNSUPPORTED
    a.dtype = _lib.FD_DTYPE_BF16
    a.head_dim = 96
    assert lib.fd_paged_decode(ctypes.byref(a), None) == _lib.FD_ERR_UNSUPPORTED
    a.head_dim, a.block_size = 128, 32
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq = 1, 6, 4, 1, 1
    assert lib.fd_paged_decode(ctypes.byref(a), None) == _lib.FD_ERR_INVALID_ARGUMENT  # 6 % 4
    r = _lib.RopeKVAppendArgs()
    r.struct_size = ctypes.sizeof(r)
    r.dtype, r.batch, r.head_dim = _lib.FD_DTYPE_BF16, 1, 128
    # neither q nor K/V rows
    assert lib.fd_rope_kv_append(ctypes.byref(r), None) == _lib.FD_ERR_INVALID_ARGUMENT
    r.rotary_dim = 3  # odd
    assert lib.fd_rope_kv_append(ctypes.byref(r), None) == _lib.FD_ERR_INVALID_ARGUMENT
    s = _lib.SplitReduceArgs()
    s.struct_size = 4
    assert lib.fd_split_kv_reduce(ctypes.byref(s), None) == _lib.FD_ERR_INVALID_ARGUMENT
    assert lib.fd_selftest_wait_timeout(0, None) == _lib.FD_ERR_INVALID_ARGUMENT
    c = _lib.CascadeArgs()
    c.struct_size = ctypes.sizeof(c)
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a)
    a.dtype, a.head_dim, a.block_size = _lib.FD_DTYPE_BF16, 128, 32
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq = 1, 8, 1, 1, 1
    a.q = a.out = a.k_cache = a.v_cache = a.block_tables = a.seq_lens = 1
    # no groups described
    assert lib.fd_cascade_decode(ctypes.byref(a), ctypes.byref(c), None) == \
        _lib.FD_ERR_INVALID_ARGUMENT
    assert lib.fd_cascade_decode(ctypes.byref(a), None, None) == _lib.FD_ERR_INVALID_ARGUMENT
    # the entry point without allocation cannot hand back partials it would
    # keep in its private static scratch: PARTIALS needs the caller's part_acc
    a.num_splits, a.epilogue = 2, _lib.FD_EPILOGUE_PARTIALS
    assert lib.fd_paged_decode_static(ctypes.byref(a), None) == _lib.FD_ERR_INVALID_ARGUMENT


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("FLASHDEC_B200_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        _lib.load_library()


def test_index_ranges_reads_all_ranges_in_one_pass():
    import torch

    from flashdec_b200 import _native

    a = torch.tensor([3, -1, 7])
    b = torch.tensor([], dtype=torch.int64)
    c = torch.tensor([5], dtype=torch.int32)
    assert _native.index_ranges(a, b, c) == [(-1, 7), None, (5, 5)]
    assert _native.index_ranges() == []
