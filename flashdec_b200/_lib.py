"""ctypes binding of ``include/flashdec_b200.h`` (libflashdec_b200.so).

The library is the only compute path: if it is missing, or the process has no
CUDA device, every entry point raises -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().with_name("libflashdec_b200.so")

FD_OK = 0
FD_ERR_INVALID_ARGUMENT = -1
FD_ERR_UNSUPPORTED = -2
FD_ERR_WORKSPACE = -3
FD_ERR_CUDA = -4
FD_ERR_ALIGNMENT = -5
FD_ERR_CAPACITY = -6
FD_STATUS_WAIT_TIMEOUT = 1
FD_STATUS_BAD_BLOCK_ID = 2

FD_DTYPE_F32 = 0
FD_DTYPE_F16 = 1
FD_DTYPE_BF16 = 2
FD_INDEX_I32 = 0
FD_INDEX_I64 = 1
FD_EPILOGUE_FUSED = 0
FD_EPILOGUE_PARTIALS = 1

_i32, _i64, _f32, _vp, _sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                              ctypes.c_void_p, ctypes.c_size_t)
_I64x2, _I64x3, _I64x4 = _i64 * 2, _i64 * 3, _i64 * 4


class PagedDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", _i32), ("dtype", _i32), ("num_seqs", _i32), ("num_q_heads", _i32),
        ("num_kv_heads", _i32), ("head_dim", _i32), ("block_size", _i32), ("num_blocks", _i32),
        ("max_blocks_per_seq", _i32), ("sm_scale", _f32),
        ("q", _vp), ("q_stride", _I64x3), ("out", _vp), ("out_stride", _I64x3),
        ("k_cache", _vp), ("k_stride", _I64x4), ("v_cache", _vp), ("v_stride", _I64x4),
        ("block_tables", _vp), ("block_tables_index", _i32), ("block_tables_stride", _I64x2),
        ("seq_lens", _vp), ("seq_lens_index", _i32), ("seq_lens_stride", _i64),
        ("append_k", _vp), ("append_k_stride", _I64x3), ("append_v", _vp),
        ("append_v_stride", _I64x3), ("slot_mapping", _vp), ("slot_mapping_index", _i32),
        ("slot_mapping_stride", _i64),
        ("num_splits", _i32), ("epilogue", _i32),
        ("part_acc", _vp), ("part_acc_stride", _I64x4), ("part_max", _vp), ("part_sum", _vp),
        ("part_stat_stride", _I64x3),
        ("tickets", _vp), ("tickets_capacity", _i64), ("scratch", _vp), ("scratch_bytes", _sz),
        ("max_ctas", _i32), ("min_tiles_per_cta", _i32),
        ("rope_dim", _i32), ("rope_inv_freq", _vp), ("rope_positions", _vp),
        ("rope_positions_index", _i32), ("rope_positions_stride", _i64),
    ]


class CascadeArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", _i32), ("num_groups", _i32), ("group_start", _vp),
        ("group_members", _vp), ("group_pages", _vp), ("seq_prefix_pages", _vp),
        ("chunks", _i32), ("tail_splits", _i32),
    ]


class SplitReduceArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", _i32), ("dtype", _i32), ("num_seqs", _i32), ("num_q_heads", _i32),
        ("head_dim", _i32), ("num_splits", _i32),
        ("part_acc", _vp), ("part_acc_stride", _I64x4), ("part_max", _vp), ("part_sum", _vp),
        ("part_stat_stride", _I64x3),
        ("seq_lens", _vp), ("seq_lens_index", _i32), ("seq_lens_stride", _i64),
        ("slot_mapping", _vp), ("slot_mapping_index", _i32), ("slot_mapping_stride", _i64),
        ("out", _vp), ("out_stride", _I64x3),
    ]


class RopeKVAppendArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", _i32), ("dtype", _i32), ("batch", _i32), ("num_q_heads", _i32),
        ("num_kv_heads", _i32), ("head_dim", _i32), ("rotary_dim", _i32), ("block_size", _i32),
        ("num_blocks", _i32), ("inv_freq", _vp),
        ("q", _vp), ("q_stride", _I64x3), ("q_out", _vp), ("q_out_stride", _I64x3),
        ("k", _vp), ("k_stride", _I64x3), ("v", _vp), ("v_stride", _I64x3),
        ("k_cache", _vp), ("k_cache_stride", _I64x4), ("v_cache", _vp),
        ("v_cache_stride", _I64x4),
        ("block_ids", _vp), ("block_offsets", _vp), ("positions", _vp),
        ("block_ids_index", _i32), ("block_offsets_index", _i32), ("positions_index", _i32),
        ("reserved", _i32),
    ]


# Exported symbols declared in include/flashdec_b200.h
EXPORTED_SYMBOLS = (
    "fd_paged_decode_workspace", "fd_paged_decode", "fd_split_kv_reduce", "fd_rope_kv_append",
    "fd_error_string", "fd_version", "fd_device_status", "fd_num_sms", "fd_paged_decode_static",
    "fd_selftest_wait_timeout", "fd_cascade_workspace", "fd_cascade_decode",
)

_lock = threading.Lock()
_lib = None
_hostpath = None


class FlashDecNativeError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""


def library_path() -> Path:
    return Path(os.environ.get("FLASHDEC_B200_LIB", str(_LIB_PATH)))


def load_library():
    """Load (once) and return the ctypes handle of libflashdec_b200.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m flashdec_b200.build` "
                "(there is no fallback implementation)"
            )
        lib = ctypes.CDLL(str(path))
        lib.fd_paged_decode_workspace.argtypes = [ctypes.POINTER(PagedDecodeArgs),
                                                  ctypes.POINTER(_sz), ctypes.POINTER(_i64)]
        lib.fd_paged_decode.argtypes = [ctypes.POINTER(PagedDecodeArgs), _vp]
        lib.fd_paged_decode_static.argtypes = [ctypes.POINTER(PagedDecodeArgs), _vp]
        lib.fd_split_kv_reduce.argtypes = [ctypes.POINTER(SplitReduceArgs), _vp]
        lib.fd_cascade_workspace.argtypes = [ctypes.POINTER(PagedDecodeArgs),
                                             ctypes.POINTER(CascadeArgs),
                                             ctypes.POINTER(ctypes.c_size_t),
                                             ctypes.POINTER(ctypes.c_int64)]
        lib.fd_cascade_decode.argtypes = [ctypes.POINTER(PagedDecodeArgs),
                                          ctypes.POINTER(CascadeArgs), _vp]
        lib.fd_rope_kv_append.argtypes = [ctypes.POINTER(RopeKVAppendArgs), _vp]
        lib.fd_error_string.argtypes = [ctypes.c_int]
        lib.fd_error_string.restype = ctypes.c_char_p
        lib.fd_version.argtypes = []
        lib.fd_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        lib.fd_num_sms.argtypes = []
        lib.fd_selftest_wait_timeout.argtypes = [ctypes.c_int64, _vp]
        for name in ("fd_paged_decode_workspace", "fd_paged_decode", "fd_paged_decode_static",
                     "fd_split_kv_reduce", "fd_selftest_wait_timeout",
                     "fd_rope_kv_append", "fd_version", "fd_device_status", "fd_num_sms"):
            getattr(lib, name).restype = ctypes.c_int
        _lib = lib
        return lib


def load_hostpath():
    """Import (once) the C++ host-path module ``_hostpath`` and point it at
    this process's library entry points.  It is built in-tree beside the
    library; a missing module raises like a missing library."""
    global _hostpath
    if _hostpath is not None:
        return _hostpath
    lib = load_library()
    with _lock:
        if _hostpath is not None:
            return _hostpath
        try:
            from . import _hostpath as hp
        except ImportError as exc:
            raise RuntimeError(
                f"flashdec_b200._hostpath is missing or does not load ({exc}): build it with "
                "`python -m flashdec_b200.build`") from exc
        if hp.ARGS_BYTES != ctypes.sizeof(PagedDecodeArgs):
            raise RuntimeError("flashdec_b200._hostpath was built against another "
                               "fd_paged_decode_args layout: rebuild it")
        hp.set_entry_points(ctypes.cast(lib.fd_paged_decode, ctypes.c_void_p).value,
                            ctypes.cast(lib.fd_cascade_decode, ctypes.c_void_p).value)
        _hostpath = hp
        return hp


def check(rc: int, what: str) -> None:
    if rc != FD_OK:
        msg = load_library().fd_error_string(rc).decode()
        raise FlashDecNativeError(f"{what} failed: {msg} (status {rc})")


def device_status(clear: bool = False) -> int:
    """Read (and optionally clear) the current device's FD_STATUS_* word (syncs)."""
    out = ctypes.c_int(0)
    check(load_library().fd_device_status(int(clear), ctypes.byref(out)), "fd_device_status")
    return out.value


def num_sms() -> int:
    n = load_library().fd_num_sms()
    if n <= 0:
        raise FlashDecNativeError("no CUDA device visible to libflashdec_b200")
    return n
