"""Marshalling from torch tensors to the C-ABI structs, and workspace reuse.

torch is used here only for device memory, the current stream and dtype
codes; every launch goes through ``libflashdec_b200.so``.
"""

from __future__ import annotations

import ctypes
import math
import threading

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.FD_DTYPE_F32, torch.float16: _lib.FD_DTYPE_F16,
               torch.bfloat16: _lib.FD_DTYPE_BF16}
_INDEX_CODE = {torch.int32: _lib.FD_INDEX_I32, torch.int64: _lib.FD_INDEX_I64}


def dtype_code(t: torch.Tensor) -> int:
    return _DTYPE_CODE[t.dtype]


def index_code(t: torch.Tensor) -> int:
    return _INDEX_CODE[t.dtype]


try:  # raw handle of the current stream without building a torch Stream object
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def stream_handle(device) -> int:
    if _raw_stream is not None:
        index = device.index if isinstance(device, torch.device) else device
        return _raw_stream(torch.cuda.current_device() if index is None else index)
    return torch.cuda.current_stream(device).cuda_stream


def strides(t: torch.Tensor, n: int):
    s = t.stride()
    if len(s) != n:
        raise ValueError(f"expected a rank-{n} tensor, got rank {len(s)}")
    return s


def index_ranges(*tensors):
    """``[(min, max), ...]`` of integer device tensors with one host
    synchronisation (one aminmax per tensor, one device-to-host read); an
    empty tensor gives ``None``."""
    parts, where = [], []
    for t in tensors:
        if t.numel() == 0:
            where.append(None)
            continue
        lo, hi = torch.aminmax(t)
        where.append(len(parts))
        parts += [lo.to(torch.int64), hi.to(torch.int64)]
    vals = torch.stack(parts).tolist() if parts else []
    return [None if w is None else (vals[w], vals[w + 1]) for w in where]


# --------------------------------------------------------------------------
# workspace: a zero-filled int32 ticket array (the kernels leave it zero) and
# fp32 scratch, grown on demand.  Every stream gets its own pair, so calls
# that overlap on the GPU (on different streams) never share tickets or
# partials; calls on one stream are ordered and share theirs.  A stream first
# seen during CUDA graph capture cannot allocate: it uses the device's default
# pair, which reserve_workspace pre-sizes and every eager call keeps at least
# as large as its own need (graphs replayed concurrently on several streams
# should therefore each be captured after an eager call on their stream).
# --------------------------------------------------------------------------
class _Workspace:
    def __init__(self):
        self.tickets = None
        self.scratch = None

    def fits(self, tickets_needed, scratch_bytes):
        return ((tickets_needed <= 0 or (self.tickets is not None
                                         and self.tickets.numel() >= tickets_needed))
                and (scratch_bytes <= 0 or (self.scratch is not None
                                            and self.scratch.numel() * 4 >= scratch_bytes)))

    def grow(self, device, tickets_needed, scratch_bytes):
        if tickets_needed > 0 and (self.tickets is None or self.tickets.numel() < tickets_needed):
            cap = max(1024, 1 << math.ceil(math.log2(tickets_needed)))
            self.tickets = torch.zeros(cap, dtype=torch.int32, device=device)
        if scratch_bytes > 0 and (self.scratch is None or self.scratch.numel() * 4 < scratch_bytes):
            n = max(1 << 16, 1 << math.ceil(math.log2((scratch_bytes + 3) // 4)))
            self.scratch = torch.empty(n, dtype=torch.float32, device=device)


_ws_lock = threading.Lock()
_ws: dict = {}  # (device index, stream handle or None for the default) -> _Workspace


def workspace(device: torch.device, tickets_needed: int, scratch_bytes: int, stream=None):
    """(tickets, scratch) for calls on `stream` (a raw handle; default: the
    current stream of `device`)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = stream_handle(idx)
    with _ws_lock:
        ws = _ws.get((idx, stream))
        if ws is not None and ws.fits(tickets_needed, scratch_bytes):
            return ws.tickets, ws.scratch
        default = _ws.setdefault((idx, None), _Workspace())
        if torch.cuda.is_current_stream_capturing():
            if ws is None and default.fits(tickets_needed, scratch_bytes):
                return default.tickets, default.scratch
            raise RuntimeError(
                "flashdec_b200 workspace must grow during CUDA graph capture; run one eager "
                "call with the largest batch first (or call reserve_workspace)"
            )
        if ws is None:
            ws = _ws[(idx, stream)] = _Workspace()
        ws.grow(device, tickets_needed, scratch_bytes)
        default.grow(device, tickets_needed, scratch_bytes)  # fallback for capture
        return ws.tickets, ws.scratch


def reserve_workspace(device, tickets: int, scratch_bytes: int) -> None:
    """Pre-size the device's default workspace (call before CUDA graph
    capture on streams that have made no eager call)."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        _ws.setdefault((idx, None), _Workspace()).grow(device, tickets, scratch_bytes)


# --------------------------------------------------------------------------
# paged decode
# --------------------------------------------------------------------------
class PreparedDecode:
    """``fd_paged_decode`` arguments prepared once for one call signature
    (shapes, strides, dtypes, scalars) together with the workspace they
    point at; :meth:`launch` only sets the data pointers (and, on a stream it
    has not launched on before, that stream's workspace).  A lock keeps two
    threads from interleaving on the shared struct (ctypes releases the GIL
    during the foreign call)."""

    __slots__ = ("lib", "args", "device", "need", "stream", "per_stream", "lock")

    def __init__(self, lib, args, device, need, stream, ws):
        self.lib = lib
        self.args = args
        self.device = device
        self.need = need  # (tickets, scratch bytes)
        self.stream = stream
        # stream -> (tickets, scratch) held, so a later growth cannot free them
        self.per_stream = {stream: ws}
        self.lock = threading.Lock()

    def _bind(self, stream):
        ws = self.per_stream.get(stream)
        if ws is None:
            ws = workspace(self.device, self.need[0], self.need[1], stream)
            self.per_stream[stream] = ws
        tickets, scratch = ws
        a = self.args
        if tickets is not None:
            a.tickets, a.tickets_capacity = tickets.data_ptr(), tickets.numel()
        if scratch is not None:
            a.scratch, a.scratch_bytes = scratch.data_ptr(), scratch.numel() * 4
        self.stream = stream

    def launch(self, q, k, v, block_tables, seq_lens, out, stream):
        a = self.args
        with self.lock:
            if stream != self.stream and (self.need[0] or self.need[1]):
                self._bind(stream)
            a.q, a.out = q.data_ptr(), out.data_ptr()
            a.k_cache, a.v_cache = k.data_ptr(), v.data_ptr()
            a.block_tables, a.seq_lens = block_tables.data_ptr(), seq_lens.data_ptr()
            rc = self.lib.fd_paged_decode(ctypes.byref(a), ctypes.c_void_p(stream))
        _lib.check(rc, "fd_paged_decode")


def prepare_paged_decode(q, k4, v4, block_tables, seq_lens, out, *, sm_scale, block_size,
                         num_seqs, num_splits=0, epilogue=_lib.FD_EPILOGUE_FUSED, append_k=None,
                         append_v=None, slot_mapping=None, partials=None, max_ctas=0,
                         min_tiles_per_cta=0, rope=None):
    """Fill the ``fd_paged_decode`` struct for these tensors and size the
    workspace; returns a :class:`PreparedDecode`.

    ``k4``/``v4`` are 4-D views in logical order [block, kv_head, token, dim]
    (any strides).  ``partials`` = (acc, max, sum) in the reference split
    workspace layout, or None for the internal workspace.  ``rope`` =
    (rotary_dim, inv_freq, positions) rotates q and ``append_k`` in the
    kernel (fused append only).
    """
    lib = _lib.load_library()
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(_lib.PagedDecodeArgs)
    a.dtype = dtype_code(q)
    a.num_seqs = int(num_seqs)
    a.num_q_heads = q.shape[1]
    a.num_kv_heads = k4.shape[1]
    a.head_dim = q.shape[2]
    a.block_size = int(block_size)
    a.num_blocks = k4.shape[0]
    a.max_blocks_per_seq = block_tables.shape[1]
    a.sm_scale = float(sm_scale)
    a.q = q.data_ptr()
    a.q_stride[:] = strides(q, 3)
    a.out = out.data_ptr()
    a.out_stride[:] = strides(out, 3)
    a.k_cache = k4.data_ptr()
    a.k_stride[:] = strides(k4, 4)
    a.v_cache = v4.data_ptr()
    a.v_stride[:] = strides(v4, 4)
    a.block_tables = block_tables.data_ptr()
    a.block_tables_index = index_code(block_tables)
    a.block_tables_stride[:] = strides(block_tables, 2)
    a.seq_lens = seq_lens.data_ptr()
    a.seq_lens_index = index_code(seq_lens)
    a.seq_lens_stride = seq_lens.stride(0)
    if append_k is not None:
        a.append_k = append_k.data_ptr()
        a.append_k_stride[:] = strides(append_k, 3)
        a.append_v = append_v.data_ptr()
        a.append_v_stride[:] = strides(append_v, 3)
        a.slot_mapping = slot_mapping.data_ptr()
        a.slot_mapping_index = index_code(slot_mapping)
        a.slot_mapping_stride = slot_mapping.stride(0)
    if rope is not None:
        rotary_dim, inv_freq, positions = rope
        a.rope_dim = int(rotary_dim)
        a.rope_inv_freq = inv_freq.data_ptr()
        a.rope_positions = positions.data_ptr()
        a.rope_positions_index = index_code(positions)
        a.rope_positions_stride = positions.stride(0)
    a.num_splits = int(num_splits)
    a.epilogue = int(epilogue)
    if partials is not None:
        acc, mx, sm = partials
        a.part_acc = acc.data_ptr()
        a.part_acc_stride[:] = strides(acc, 4)
        a.part_max = mx.data_ptr()
        a.part_sum = sm.data_ptr()
        a.part_stat_stride[:] = strides(mx, 3)
    a.max_ctas = int(max_ctas)
    a.min_tiles_per_cta = int(min_tiles_per_cta)
    scratch_bytes = ctypes.c_size_t(0)
    tickets_needed = ctypes.c_int64(0)
    _lib.check(lib.fd_paged_decode_workspace(ctypes.byref(a), ctypes.byref(scratch_bytes),
                                             ctypes.byref(tickets_needed)),
               "fd_paged_decode_workspace")
    ws = (None, None)
    stream = stream_handle(q.device)
    if scratch_bytes.value or tickets_needed.value:
        ws = tickets, scratch = workspace(q.device, tickets_needed.value, scratch_bytes.value,
                                          stream)
        if tickets is not None:
            a.tickets = tickets.data_ptr()
            a.tickets_capacity = tickets.numel()
        if scratch is not None:
            a.scratch = scratch.data_ptr()
            a.scratch_bytes = scratch.numel() * 4
    return PreparedDecode(lib, a, q.device, (tickets_needed.value, scratch_bytes.value), stream,
                          ws)


def paged_decode(q, k4, v4, block_tables, seq_lens, out, **kw):
    """Prepare and launch ``fd_paged_decode`` on the current stream; returns
    ``out``.  Keyword arguments as :func:`prepare_paged_decode`."""
    prep = prepare_paged_decode(q, k4, v4, block_tables, seq_lens, out, **kw)
    a = prep.args
    _lib.check(prep.lib.fd_paged_decode(ctypes.byref(a),
                                        ctypes.c_void_p(stream_handle(q.device))),
               "fd_paged_decode")
    return out


class CascadeGroups:
    """Shared-prefix groups of a batch for ``fd_cascade_decode``: ``groups``
    lists the sequence indices (rows of q) of each group and ``pages`` its
    shared leading pages (the same physical pages at the start of every
    member's block-table row; ``pages * block_size`` a multiple of 32).  The
    group description stays in host memory (the C-ABI copies it into the
    launch); the per-sequence prefix pages go to the device once."""

    MAX_GROUPS = 32
    MAX_MEMBERS = 512

    def __init__(self, groups, pages, num_seqs, block_size, device):
        if len(groups) != len(pages) or not groups:
            raise ValueError("one page count per group, at least one group")
        start = [0]
        members = []
        seq_pages = [0] * int(num_seqs)
        for g, pg in zip(groups, pages):
            if int(pg) <= 0 or (int(pg) * int(block_size)) % 32:
                raise ValueError("shared prefix tokens must be a positive multiple of 32")
            if not g:
                raise ValueError("a group needs at least one member")
            for b in g:
                if not 0 <= int(b) < num_seqs or seq_pages[int(b)]:
                    raise ValueError("group members must be distinct rows of the batch")
                seq_pages[int(b)] = int(pg)
            members += [int(b) for b in g]
            start.append(len(members))
        if len(groups) > self.MAX_GROUPS or len(members) > self.MAX_MEMBERS:
            raise ValueError(f"at most {self.MAX_GROUPS} groups and {self.MAX_MEMBERS} members")
        self.host_start = (ctypes.c_int32 * len(start))(*start)
        self.host_members = (ctypes.c_int32 * len(members))(*members)
        self.host_pages = (ctypes.c_int32 * len(pages))(*[int(x) for x in pages])
        seq = torch.tensor(seq_pages, dtype=torch.int32)
        self.seq_pages = seq.pin_memory().to(device, non_blocking=True) \
            if torch.device(device).type == "cuda" else seq
        a = self.args = _lib.CascadeArgs()
        a.struct_size = ctypes.sizeof(_lib.CascadeArgs)
        a.num_groups = len(groups)
        a.group_start = ctypes.addressof(self.host_start)
        a.group_members = ctypes.addressof(self.host_members)
        a.group_pages = ctypes.addressof(self.host_pages)
        a.seq_prefix_pages = self.seq_pages.data_ptr()


def cascade_workspace(decode_args, cascade_args):
    """(scratch bytes, ticket entries) ``fd_cascade_decode`` needs."""
    lib = _lib.load_library()
    nbytes = ctypes.c_size_t(0)
    tickets = ctypes.c_int64(0)
    _lib.check(lib.fd_cascade_workspace(ctypes.byref(decode_args), ctypes.byref(cascade_args),
                                        ctypes.byref(nbytes), ctypes.byref(tickets)),
               "fd_cascade_workspace")
    return nbytes.value, tickets.value


def cascade_decode(q, k4, v4, block_tables, seq_lens, out, groups, *, sm_scale, block_size,
                   num_seqs, chunks=0, tail_splits=0, append_k=None, append_v=None,
                   slot_mapping=None, rope=None):
    """Launch ``fd_cascade_decode`` (prefix pass, then the tail pass with the
    merge) on the current stream; ``groups`` is a :class:`CascadeGroups`.
    Returns ``out``."""
    prep = prepare_paged_decode(q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale,
                                block_size=block_size, num_seqs=num_seqs, num_splits=1,
                                append_k=append_k, append_v=append_v,
                                slot_mapping=slot_mapping, rope=rope)
    a = prep.args
    c = groups.args
    c.chunks, c.tail_splits = int(chunks), int(tail_splits)
    nbytes, ntickets = cascade_workspace(a, c)
    tickets, scratch = workspace(q.device, ntickets, nbytes)
    a.scratch, a.scratch_bytes = scratch.data_ptr(), scratch.numel() * 4
    a.tickets, a.tickets_capacity = tickets.data_ptr(), tickets.numel()
    _lib.check(prep.lib.fd_cascade_decode(ctypes.byref(a), ctypes.byref(c),
                                          ctypes.c_void_p(stream_handle(q.device))),
               "fd_cascade_decode")
    return out


def split_kv_reduce(acc, mx, sm, seq_lens, out, *, num_seqs, slot_mapping=None):
    lib = _lib.load_library()
    a = _lib.SplitReduceArgs()
    a.struct_size = ctypes.sizeof(_lib.SplitReduceArgs)
    a.dtype = dtype_code(out)
    a.num_seqs = int(num_seqs)
    a.num_q_heads = out.shape[1]
    a.head_dim = out.shape[2]
    a.num_splits = acc.shape[2]
    a.part_acc = acc.data_ptr()
    a.part_acc_stride[:] = strides(acc, 4)
    a.part_max = mx.data_ptr()
    a.part_sum = sm.data_ptr()
    a.part_stat_stride[:] = strides(mx, 3)
    a.seq_lens = seq_lens.data_ptr()
    a.seq_lens_index = index_code(seq_lens)
    a.seq_lens_stride = seq_lens.stride(0)
    if slot_mapping is not None:
        a.slot_mapping = slot_mapping.data_ptr()
        a.slot_mapping_index = index_code(slot_mapping)
        a.slot_mapping_stride = slot_mapping.stride(0)
    a.out = out.data_ptr()
    a.out_stride[:] = strides(out, 3)
    _lib.check(lib.fd_split_kv_reduce(ctypes.byref(a), ctypes.c_void_p(stream_handle(out.device))),
               "fd_split_kv_reduce")
    return out


def rope_kv_append(q, q_out, k, v, k_cache4, v_cache4, block_ids, block_offsets, positions,
                   rotary_dim, inv_freq):
    """Launch fd_rope_kv_append; q/q_out may be None (K/V only) and k may be
    None (rotate q only: v, the caches and block ids/offsets are then unused)."""
    lib = _lib.load_library()
    a = _lib.RopeKVAppendArgs()
    a.struct_size = ctypes.sizeof(_lib.RopeKVAppendArgs)
    lead = k if k is not None else q
    a.dtype = dtype_code(lead)
    a.batch = lead.shape[0]
    a.head_dim = lead.shape[2]
    a.rotary_dim = int(rotary_dim)
    if inv_freq is not None:
        a.inv_freq = inv_freq.data_ptr()
    if q is not None:
        a.num_q_heads = q.shape[1]
        a.q = q.data_ptr()
        a.q_stride[:] = strides(q, 3)
        a.q_out = q_out.data_ptr()
        a.q_out_stride[:] = strides(q_out, 3)
    if k is not None:
        a.num_kv_heads = k.shape[1]
        a.block_size = k_cache4.shape[2]
        a.num_blocks = k_cache4.shape[0]
        a.k = k.data_ptr()
        a.k_stride[:] = strides(k, 3)
        a.v = v.data_ptr()
        a.v_stride[:] = strides(v, 3)
        a.k_cache = k_cache4.data_ptr()
        a.k_cache_stride[:] = strides(k_cache4, 4)
        a.v_cache = v_cache4.data_ptr()
        a.v_cache_stride[:] = strides(v_cache4, 4)
        a.block_ids = block_ids.data_ptr()
        a.block_offsets = block_offsets.data_ptr()
        a.block_ids_index = index_code(block_ids)
        a.block_offsets_index = index_code(block_offsets)
    if positions is not None:
        a.positions = positions.data_ptr()
        a.positions_index = index_code(positions)
    _lib.check(lib.fd_rope_kv_append(ctypes.byref(a),
                                     ctypes.c_void_p(stream_handle(lead.device))),
               "fd_rope_kv_append")


# --------------------------------------------------------------------------
# RoPE frequency tables, computed once per (rotary_dim, base) on the host with
# the reference formula (flashdec/rope.py:66-67: fp32 arange, fp32 division,
# fp32 torch.pow) and kept on each device.
# --------------------------------------------------------------------------
_freq_lock = threading.Lock()
_freq_host: dict = {}
_freq_dev: dict = {}


def inv_freq_host(rotary_dim: int, base: float) -> torch.Tensor:
    key = (int(rotary_dim), float(base))
    with _freq_lock:
        t = _freq_host.get(key)
        if t is None:
            steps = torch.arange(0, rotary_dim, 2, dtype=torch.float32)
            t = torch.pow(float(base), -steps / rotary_dim).contiguous()
            _freq_host[key] = t
        return t


def inv_freq_device(rotary_dim: int, base: float, device) -> torch.Tensor:
    device = torch.device(device)
    key = (int(rotary_dim), float(base), device.index)
    with _freq_lock:
        t = _freq_dev.get(key)
    if t is None:
        host = inv_freq_host(rotary_dim, base)
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("RoPE table not resident on the device; run once before capture")
        t = host.to(device)
        with _freq_lock:
            _freq_dev[key] = t
    return t
