"""Paged KV cache for B200 decode: the reference ``PagedKVCache`` API.

Drop-in for ``flashdec/cache.py`` (cysong2025/flashdec).  Storage is
``[num_layers, max_blocks, num_kv_heads, block_size, head_dim]`` (token-major
pages, :136-145).  Every integer decision lives in :class:`BlockLedger`
(bit-exact with the reference's allocator); every data write goes through the
C-ABI kernels of ``libflashdec_b200.so`` (``fd_rope_kv_append``), so data
methods need a CUDA-resident cache and raise otherwise -- there is no CPU
write path.

Transaction metadata (positions, physical block ids, offsets, effective
sequence lengths, block table) is uploaded to the device once per
transaction at ``begin_token`` and reused by every layer; the reference
rebuilds those tensors on every layer write (cache.py:592, :1043-1076).
"""

from __future__ import annotations

import ctypes
import itertools
import math
import os
from dataclasses import dataclass, replace
from typing import Hashable

import numpy as np
import torch

from . import _native
from .ledger import BlockLedger


@dataclass(frozen=True)
class KVTokenTransactionView:
    """Detached public snapshot of one multi-layer token transaction."""

    transaction_id: int
    cache_version: int
    request_ids: tuple
    positions: object
    physical_block_ids: object
    block_offsets: object
    block_tables: object
    effective_seq_lens: object
    next_layer_idx: int
    state: str


class _PinnedStaging:
    """Reused pinned host memory for the per-token metadata uploads.

    ``tensor.pin_memory()`` per upload asks torch's caching host allocator for
    a block, and its blocks are released only once their copy has completed:
    with the device a few steps behind the host (the normal state of a decode
    loop) every upload pins new memory, which costs about 100 us.  Here one
    pinned arena of ``slots`` equal slots is allocated up front and its slots
    are rewritten in turn; before a slot is reused the host waits for the
    event recorded after that slot's last copy (normally long complete).  The
    wait, the copy and the event live in the C++ host path.  An upload larger
    than a slot re-allocates the arena with larger slots (after every pending
    copy of the old one has completed)."""

    _ids = itertools.count(1)

    def __init__(self, slots=64):
        from . import _lib

        self.hp = _lib.load_hostpath()
        self.ring = next(self._ids)
        self.slots = slots
        self.slot_bytes = 0
        self.arena = None
        self.host = None
        self.base = 0
        self.next = 0

    def __del__(self):
        try:
            self.hp.staging_release(self.ring)
        except Exception:  # interpreter shutdown
            pass

    def _grow(self, nbytes):
        for i in range(self.slots if self.arena is not None else 0):
            self.hp.staging_wait(self.ring, self.slots, i)
        size = max(16384, 1 << (nbytes - 1).bit_length())
        self.arena = torch.empty(self.slots * size, dtype=torch.uint8, pin_memory=True)
        self.host = self.arena.numpy()
        self.base = self.arena.data_ptr()
        self.slot_bytes = size
        self.next = 0

    def upload(self, array, device):
        """Device copy (uint8, on the device's current stream) of a numpy array."""
        if torch._C._cuda_getDevice() != device.index:
            with torch.cuda.device(device):
                return self.upload(array, device)
        raw = np.ascontiguousarray(array).reshape(-1).view(np.uint8)
        n = raw.size
        if n > self.slot_bytes:
            self._grow(n)
        i = self.next
        self.next = (i + 1) % self.slots
        self.hp.staging_wait(self.ring, self.slots, i)
        off = i * self.slot_bytes
        self.host[off:off + n] = raw
        return self.hp.staging_copy(self.ring, self.slots, i, self.base + off, n)


class _DeviceMeta:
    """Device copies of one transaction's metadata: ``kernel`` tensors are
    private (the kernels read only these), ``public`` ones back the views.

    The per-token integers (positions, block ids, offsets and slots
    ``block_id * block_size + offset`` as int64, the effective lengths as
    int32) travel as one packed byte buffer: one pinned staging copy, one
    host-to-device copy.  The block table comes from
    :class:`_BlockTableCache` and is shared with earlier transactions while
    its rows are unchanged."""

    def __init__(self, device, positions, locations, table, block_size, cascade=None,
                 staging=None):
        n = len(positions)
        self.cascade = cascade  # _native.CascadeGroups of the batch's shared prefixes, or None
        packed = np.empty(4 * n * 8 + n * 4, np.uint8)
        i64 = packed[:4 * n * 8].view(np.int64)
        i64[:n] = positions
        i64[n:2 * n] = [b for b, _ in locations]
        i64[2 * n:3 * n] = [o for _, o in locations]
        i64[3 * n:] = i64[n:2 * n] * block_size + i64[2 * n:3 * n]
        packed[4 * n * 8:].view(np.int32)[:] = i64[:n] + 1
        if device.type == "cuda":
            buf = staging.upload(packed, device)
            self._unpack = staging.hp.unpack_meta
        else:
            buf = torch.from_numpy(packed)
            self._unpack = _unpack_meta
        self._packed, self.block_tables = buf, table
        (self.positions, self.block_ids, self.offsets, self.slots,
         self.eff_seq_lens) = self._unpack(buf, n)
        self._public = None

    @property
    def public(self):
        """The transaction's public metadata: one copy per token, taken on
        first use (kernels read the internal buffers, which callers never
        see)."""
        pub = self._public
        if pub is None:
            pub = self._public = self.snapshot()
        return pub

    def snapshot(self):
        """Fresh copies of the metadata (two copies: packed integers, table)."""
        pub = self._unpack(self._packed.clone(), len(self.positions))
        return dict(positions=pub[0], physical_block_ids=pub[1], block_offsets=pub[2],
                    effective_seq_lens=pub[4], block_tables=self.block_tables.clone())


def _unpack_meta(buf, n):
    """(positions, block ids, offsets, slots) int64 and effective lengths
    int32 views of a packed metadata buffer."""
    pos, bid, off, slot = buf[:4 * n * 8].view(torch.int64).view(4, n).unbind(0)
    return pos, bid, off, slot, buf[4 * n * 8:].view(torch.int32)


class _BlockTableCache:
    """Block table of the last transaction, kept on the device.

    Decode steps usually repeat the same request rows and a row only changes
    when its request takes a new block (once per ``block_size`` tokens), so
    rebuilding the padded table from Python lists every step would dominate
    ``begin_token``.  Rows are compared against copies of the ledger's lists
    (exact), changed rows are patched into a copy of the previous host array,
    and an unchanged table is reused as is: a table is never written after
    its upload, so transactions may share it."""

    def __init__(self):
        self.ids = None
        self.rows = None
        self.host = None
        self.table = None

    def get(self, device, ids, block_lists, staging=None):
        n = len(block_lists)
        width = max(1, max(map(len, block_lists)))
        if self.ids == ids and self.host is not None and self.host.shape[1] == width:
            changed = [i for i, (a, b) in enumerate(zip(block_lists, self.rows)) if a != b]
            if not changed:
                return self.table
            host = self.host.copy()
        else:
            changed = range(n)
            host = np.empty((n, width), np.int32)
        for i in changed:
            row = block_lists[i]
            host[i, :len(row)] = row
            host[i, len(row):] = -1
        if device.type == "cuda":
            table = staging.upload(host, device).view(torch.int32).view(host.shape)
        else:
            table = torch.from_numpy(host).clone()
        self.ids, self.rows, self.host, self.table = ids, [list(b) for b in block_lists], host, table
        return table


def _cascade_enabled():
    # Opt-in: on the Qwen c5 shape (16 rows sharing 4096 tokens) the prefix
    # pass + tail pass measure 28-34 us per layer against 24 us for the plain
    # decode, whose shared-page re-reads hit L2; the prefix pass is bound by
    # mma.sync latency, not by memory.
    return os.environ.get("FLASHDEC_B200_CASCADE", "0") == "1"


class _CascadeCache:
    """Shared-prefix groups of the last transaction's rows (device copy).

    Rows of one transaction whose requests are attached to the same
    registered prefix start their block tables with the same physical pages
    (``shared_block_count`` of them).  With FLASHDEC_B200_CASCADE=1, groups
    of at least two rows with at least 128 shared tokens go to
    ``fd_cascade_decode``; the shared length is
    rounded down to whole 32-token tiles (the rest is read as private
    tokens).  The description only changes when the rows or their prefixes
    do, so it is rebuilt only then."""

    MIN_MEMBERS = 2
    MIN_TOKENS = 128

    def __init__(self):
        self.key = None
        self.groups = None

    def get(self, device, ids, requests, block_size):
        attached = tuple((requests[r].prefix_id, requests[r].shared_block_count) for r in ids)
        key = (ids, attached)
        if key == self.key:
            return self.groups
        unit = 32 // math.gcd(32, block_size)  # pages per 32-token tile
        by_prefix = {}
        for row, (pid, count) in enumerate(attached):
            if pid is not None and count > 0:
                by_prefix.setdefault(pid, (count, []))[1].append(row)
        rows, pages = [], []
        for count, members in by_prefix.values():
            shared = (count // unit) * unit
            if len(members) >= self.MIN_MEMBERS and shared * block_size >= self.MIN_TOKENS:
                rows.append(members)
                pages.append(shared)
        self.groups = (_native.CascadeGroups(rows, pages, len(ids), block_size, device)
                       if rows else None)
        self.key = key
        return self.groups


class _FusedLayerLauncher:
    """Launch state of the engine's fused layer step for one open token.

    A layer is ONE ``fd_paged_decode`` launch (``fd_cascade_decode`` when rows
    share a registered prefix: see :class:`_CascadeCache`) with the fused
    append and RoPE fields set: the kernel rotates q and the new K row by the transaction's
    positions, stores the rotated K and the raw V row at the reserved slot
    (``block_id * block_size + offset``) and attends over the sequence with
    that row -- the same arithmetic as ``fd_rope_kv_append`` followed by
    ``fd_paged_decode`` (one shared rotation routine; bit-identical caches and
    outputs).  The argument struct is filled once per transaction from the
    cache-owned device metadata and the per-device decode workspace; a layer
    only sets its q/k/v/output pointers and the layer's cache planes.
    """

    def __init__(self, cache, meta, num_q_heads, sm_scale):
        from . import _lib

        self.lib = _lib.load_library()
        self.check = _lib.check
        n = meta.positions.numel()
        hkv, d, bs = cache.num_kv_heads, cache.head_dim, cache.block_size
        self.device = cache.device
        self.qshape = (n, num_q_heads, d)
        self.kvshape = (n, hkv, d)
        kc, vc = cache.k_cache, cache.v_cache
        esz = kc.element_size()
        self.k_base, self.v_base = kc.data_ptr(), vc.data_ptr()
        self.k_layer_bytes = kc.stride(0) * esz
        self.v_layer_bytes = vc.stride(0) * esz
        q_strides = (num_q_heads * d, d, 1)
        kv_strides = (hkv * d, d, 1)
        self.rope_key = None
        self.rope_args = None  # last (rotary_dim, base) as given, and its checked form
        self.rope_checked = None

        da = _lib.PagedDecodeArgs()
        da.struct_size = ctypes.sizeof(da)
        da.dtype = _native.dtype_code(kc)
        da.num_seqs = n
        da.num_q_heads = num_q_heads
        da.num_kv_heads = hkv
        da.head_dim = d
        da.block_size = bs
        da.num_blocks = cache.max_blocks
        da.max_blocks_per_seq = meta.block_tables.shape[1]
        da.sm_scale = float(sm_scale if sm_scale is not None else d ** -0.5)
        da.q_stride[:] = q_strides
        da.out_stride[:] = q_strides
        da.k_stride[:] = kc.stride()[1:]
        da.v_stride[:] = vc.stride()[1:]
        da.block_tables = meta.block_tables.data_ptr()
        da.block_tables_index = _lib.FD_INDEX_I32
        da.block_tables_stride[:] = meta.block_tables.stride()
        da.seq_lens = meta.eff_seq_lens.data_ptr()
        da.seq_lens_index = _lib.FD_INDEX_I32
        da.seq_lens_stride = 1
        da.append_k_stride[:] = kv_strides
        da.append_v_stride[:] = kv_strides
        da.slot_mapping = meta.slots.data_ptr()
        da.slot_mapping_index = _lib.FD_INDEX_I64
        da.slot_mapping_stride = 1
        da.rope_positions = meta.positions.data_ptr()
        da.rope_positions_index = _lib.FD_INDEX_I64
        da.rope_positions_stride = 1
        da.epilogue = _lib.FD_EPILOGUE_FUSED
        # the plan (and so the workspace need) depends on shapes only
        da.q = da.out = da.k_cache = da.v_cache = da.append_k = da.append_v = 1
        scratch = ctypes.c_size_t(0)
        tickets = ctypes.c_int64(0)
        self.cascade = meta.cascade
        if self.cascade is not None:
            # shared prefixes: prefix pass, then the tail pass with the merge
            scratch.value, tickets.value = _native.cascade_workspace(da, self.cascade.args)
        else:
            self.check(self.lib.fd_paged_decode_workspace(ctypes.byref(da), ctypes.byref(scratch),
                                                          ctypes.byref(tickets)),
                       "fd_paged_decode_workspace")
        self.workspace = (None, None)
        if scratch.value or tickets.value:
            # held here so that a later growth of the shared per-device
            # workspace cannot free the buffers this transaction points at
            t, s = self.workspace = _native.workspace(self.device, tickets.value, scratch.value)
            if t is not None:
                da.tickets, da.tickets_capacity = t.data_ptr(), t.numel()
            if s is not None:
                da.scratch, da.scratch_bytes = s.data_ptr(), s.numel() * 4
        self.da = da
        # the C++ host path runs each layer on these structs (kept alive here)
        self.hostpath = _lib.load_hostpath()
        self.da_addr = ctypes.addressof(da)
        self.cascade_addr = (ctypes.addressof(self.cascade.args)
                             if self.cascade is not None else 0)

    def _set_rope(self, rotary_dim, base):
        key = (rotary_dim, base)
        if key != self.rope_key:
            self.da.rope_dim = rotary_dim
            self.da.rope_inv_freq = _native.inv_freq_device(rotary_dim, base,
                                                            self.device).data_ptr()
            self.rope_key = key

    def run(self, layer_idx, q, k, v, rotary_dim, base):
        """RoPE + K/V store + decode in one launch; returns the output.

        The C++ host path checks that q, k and v are contiguous and match
        the transaction's shapes (ValueError otherwise), allocates the
        output, sets the layer's pointers and launches on the current
        stream."""
        if (rotary_dim, base) != self.rope_key:
            self._set_rope(rotary_dim, base)
        out = self.hostpath.layer_run(self.da_addr, self.cascade_addr, q, k, v,
                                      self.k_base + layer_idx * self.k_layer_bytes,
                                      self.v_base + layer_idx * self.v_layer_bytes)
        if type(out) is int:
            self.check(out, "fd_cascade_decode" if self.cascade_addr else "fd_paged_decode")
        return out


class PagedKVCache:
    """Fixed-block KV cache runtime for single-token decode (see module doc)."""

    ACTIVE = BlockLedger.ACTIVE
    FINISHED = BlockLedger.FINISHED
    CANCELLED = BlockLedger.CANCELLED
    _TERMINAL_TRANSACTION_HISTORY_LIMIT = BlockLedger.TERMINAL_HISTORY_LIMIT

    def __init__(self, num_layers, num_kv_heads, head_dim, block_size, max_blocks, dtype=None,
                 device=None, prefix_cache_capacity_blocks=0):
        if dtype is None:
            dtype = torch.float16
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        for name, value in [("num_layers", num_layers), ("num_kv_heads", num_kv_heads),
                            ("head_dim", head_dim), ("block_size", block_size),
                            ("max_blocks", max_blocks)]:
            if int(value) <= 0:
                raise ValueError(f"{name} must be positive")
        if not torch.empty((), dtype=dtype).is_floating_point():
            raise ValueError("dtype must be a floating point torch dtype")
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.block_size = int(block_size)
        self.max_blocks = int(max_blocks)
        self._ledger = BlockLedger(self.num_layers, self.block_size, self.max_blocks,
                                   prefix_cache_capacity_blocks)
        self.prefix_cache_capacity_blocks = self._ledger.prefix_cache_capacity_blocks
        self.dtype = dtype
        shape = (self.num_layers, self.max_blocks, self.num_kv_heads, self.block_size,
                 self.head_dim)
        self.k_cache = torch.zeros(shape, device=device, dtype=dtype)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.device = self.k_cache.device
        self._tables = _BlockTableCache()
        self._staging_ring = None  # _PinnedStaging, created by the first CUDA upload
        self._cascades = _CascadeCache()

    # ----------------------------------------------------------- lifecycle
    def add_request(self, request_id):
        self._ledger.add_request(request_id)
        return self

    def finish_request(self, request_id):
        return self._ledger.close_request(request_id, self.FINISHED)

    def cancel_request(self, request_id):
        return self._ledger.close_request(request_id, self.CANCELLED)

    def request_state(self, request_id):
        st = self._ledger.require_request(request_id)
        return {"request_id": request_id, "status": st.status, "seq_len": st.seq_len,
                "block_ids": tuple(st.block_ids), "prefix_id": st.prefix_id,
                "shared_block_count": st.shared_block_count}

    def request_block_ids(self, request_id):
        return tuple(self._ledger.require_request(request_id).block_ids)

    def next_positions(self, request_ids, device=None):
        ids = self._normalize_request_ids(request_ids)
        if not ids:
            raise ValueError("request_ids must be non-empty")
        if len(set(ids)) != len(ids):
            raise ValueError("request_ids must be unique")
        return torch.tensor(self._ledger.next_positions(ids),
                            device=device if device is not None else self.device,
                            dtype=torch.int64)

    # -------------------------------------------------------------- prefix
    def register_prefix(self, prefix_id, k_blocks, v_blocks):
        """Copy immutable full K/V blocks ``[L, n, Hkv, bs, D]`` into the
        shared-prefix registry (evicting inactive LRU prefixes if needed)."""
        if self._ledger.open_transaction_id is not None:
            raise RuntimeError("cannot register a prefix during an open token transaction")
        BlockLedger.check_prefix_id(prefix_id)
        if prefix_id in self._ledger.prefixes:
            raise RuntimeError(f"prefix_id {prefix_id!r} is already registered")
        k_blocks, v_blocks = self._prepare_prefix_blocks(k_blocks, v_blocks)
        block_ids = self._ledger.register_prefix(prefix_id, int(k_blocks.shape[1]))
        index = torch.tensor(block_ids, device=self.device, dtype=torch.long)
        self.k_cache.index_copy_(1, index, k_blocks)
        self.v_cache.index_copy_(1, index, v_blocks)
        self._ledger.publish_prefix(prefix_id, block_ids)
        return self.prefix_state(prefix_id)

    def attach_prefix(self, request_id, prefix_id):
        return self._ledger.attach_prefix(request_id, prefix_id)

    def evict_prefix(self, prefix_id):
        return self._ledger.evict_prefix(prefix_id)

    def prefix_state(self, prefix_id):
        return self._ledger.prefix_state(prefix_id)

    # ------------------------------------------------------- legacy append
    def append(self, layer_idx, request_ids, k, v):
        """Append one token of K/V per request (single-layer caches).

        Returns the padded block table of ``request_ids`` (int32, pad -1)."""
        return self._legacy_append(layer_idx, request_ids, k, v)

    def append_cuda(self, layer_idx, request_ids, k, v):
        """Same as :meth:`append` (both use the native copy kernel)."""
        return self._legacy_append(layer_idx, request_ids, k, v)

    def _legacy_append(self, layer_idx, request_ids, k, v):
        self._ledger.require_legacy_append_available()
        layer_idx, ids, k, v = self._prepare_append_inputs(layer_idx, request_ids, k, v)
        self._require_cuda("append")
        if not k.is_contiguous() or not v.is_contiguous():
            raise ValueError("append_cuda requires contiguous k and v tensors")
        self._ledger.preflight_append(ids)
        locations = self._ledger.allocate_append_locations(ids)
        bid = torch.tensor([b for b, _ in locations], dtype=torch.int64).to(self.device)
        off = torch.tensor([o for _, o in locations], dtype=torch.int64).to(self.device)
        with torch.cuda.device(self.device):
            _native.rope_kv_append(None, None, k, v, self.k_cache[layer_idx],
                                   self.v_cache[layer_idx], bid, off, None, 0, None)
        self._ledger.advance_lengths(ids)
        return self.block_tables(ids)

    def append_fused_cuda(self, layer_idx, request_ids, q, k, v, positions, rotary_dim=None,
                          base=10_000.0):
        """Fused RoPE + append at allocator-chosen slots; returns
        ``(rotated_q, block_tables)`` (reference cache.py:353-433)."""
        from ._fused_rope_kv_append import _fused_rope_kv_append_trusted

        self._ledger.require_legacy_append_available()
        layer_idx, ids, k, v = self._prepare_append_inputs(layer_idx, request_ids, k, v)
        self._require_cuda("append_fused_cuda")
        if self.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError("append_fused_cuda supports cache dtype float16, bfloat16, or float32")
        if q.dim() != 3 or q.shape[0] != len(ids) or q.shape[1] <= 0 or q.shape[2] != self.head_dim:
            raise ValueError("q shape must match request count and cache head_dim")
        if q.device != self.device or q.dtype != self.dtype:
            raise ValueError("q must use the cache device and dtype")
        if positions.dim() != 1 or positions.numel() != len(ids):
            raise ValueError("positions must have shape [num_requests]")
        if positions.device != self.device or positions.dtype not in (torch.int32, torch.int64):
            raise ValueError("positions must use int32/int64 on the cache device")
        if bool(torch.any(positions < 0).item()):
            raise ValueError("positions must be non-negative")
        rotary_dim = self._check_rope_args(rotary_dim, base)
        if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
            raise ValueError("append_fused_cuda requires contiguous q, k, and v tensors")
        self._ledger.preflight_append(ids)
        locations = self._ledger.allocate_append_locations(ids)
        bid = torch.tensor([b for b, _ in locations], dtype=torch.int64).to(self.device)
        off = torch.tensor([o for _, o in locations], dtype=torch.int64).to(self.device)
        q_rot = _fused_rope_kv_append_trusted(q, k, v, self.k_cache[layer_idx],
                                              self.v_cache[layer_idx], bid, off,
                                              positions.to(torch.int64), rotary_dim=rotary_dim,
                                              base=base)
        self._ledger.advance_lengths(ids)
        return q_rot, self.block_tables(ids)

    def _staging(self):
        if self.device.type != "cuda":
            return None
        if self._staging_ring is None:
            self._staging_ring = _PinnedStaging()
        return self._staging_ring

    # --------------------------------------------------------- transactions
    def begin_token(self, request_ids):
        """Reserve one token location per request for every layer; seq_len is
        published once at :meth:`commit_token`."""
        ids = tuple(self._normalize_request_ids(request_ids))
        tx = self._ledger.begin_token(ids)
        try:
            table = self._tables.get(self.device, ids,
                                     [self._ledger.requests[r].block_ids for r in ids],
                                     self._staging())
            cascade = (self._cascades.get(self.device, ids, self._ledger.requests,
                                          self.block_size)
                       if self.device.type == "cuda" and _cascade_enabled() else None)
            tx.device_view = _DeviceMeta(self.device, tx.positions, tx.locations, table,
                                         self.block_size, cascade, self._staging())
        except Exception:
            self._ledger.abort_token(tx)
            raise
        return self._view(tx)

    def write_token_layer(self, transaction, layer_idx, k, v):
        """Write one layer's K/V at the locations reserved by begin_token."""
        state = self._require_open_transaction(transaction)
        try:
            layer_idx, k, v = self._prepare_transaction_layer_write(state, layer_idx, k, v)
            self._require_cuda("write_token_layer")
            meta = state.device_view
            with torch.cuda.device(self.device):
                _native.rope_kv_append(None, None, k, v, self.k_cache[layer_idx],
                                       self.v_cache[layer_idx], meta.block_ids, meta.offsets,
                                       None, 0, None)
        except Exception:
            self._ledger.transaction_failure_count += 1
            raise
        self._ledger.record_layer_write(state, layer_idx)
        return self._view(state)

    def write_token_layer_fused_cuda(self, transaction, layer_idx, q, k, v, *, rotary_dim=None,
                                     base=10_000.0):
        """Fused RoPE + K/V write of one layer at the reserved locations;
        returns ``(rotated_q, view)``.  The kernel reads the cache-owned
        device metadata of the open transaction, never caller tensors."""
        state = self._require_open_transaction(transaction)
        try:
            q_rot = self._fused_layer_write(state, layer_idx, q, k, v, rotary_dim, base)
        except Exception:
            self._ledger.transaction_failure_count += 1
            raise
        self._ledger.record_layer_write(state, int(layer_idx))
        return q_rot, self._view(state)

    def _fused_layer_write(self, state, layer_idx, q, k, v, rotary_dim, base, q_out=None):
        from ._fused_rope_kv_append import _fused_rope_kv_append_trusted

        layer_idx, k, v = self._prepare_transaction_layer_write(state, layer_idx, k, v)
        self._require_cuda("write_token_layer_fused_cuda")
        if self.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError("write_token_layer_fused_cuda supports float16, bfloat16, or float32")
        if q.dim() != 3 or q.shape[0] != len(state.request_ids):
            raise ValueError("q shape must match transaction request count and cache head_dim")
        if q.shape[1] <= 0 or q.shape[2] != self.head_dim:
            raise ValueError("q shape must match transaction request count and cache head_dim")
        if q.device != self.device or q.dtype != self.dtype:
            raise ValueError("q must use the cache device and dtype")
        if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
            raise ValueError("write_token_layer_fused_cuda requires contiguous q, k, and v tensors")
        meta = state.device_view
        return _fused_rope_kv_append_trusted(q, k, v, self.k_cache[layer_idx],
                                             self.v_cache[layer_idx], meta.block_ids,
                                             meta.offsets, meta.positions, rotary_dim=rotary_dim,
                                             base=base, q_out=q_out)

    def _fused_layer_step(self, transaction, layer_idx, q, k, v, rotary_dim, base, sm_scale):
        """Engine fast path of one layer, one launch: RoPE of q and K, K/V
        store at the reserved slots and paged decode over the transaction's
        block tables and effective lengths.  Returns ``(output, public
        metadata)``; the launch arguments are prepared once per transaction
        (:class:`_FusedLayerLauncher`)."""
        # The engine has already checked q/k/v (tensors, shapes, device,
        # dtype); this adds the transaction, layer order, contiguity (in
        # run) and RoPE argument checks.
        state = self._require_open_transaction(transaction)
        try:
            layer_idx = self._ledger.check_layer_for_write(state, layer_idx)
            meta = state.device_view
            key = (int(q.shape[1]), sm_scale)
            launcher = getattr(meta, "launcher", None)
            if launcher is None or meta.launcher_key != key:
                self._require_cuda("write_token_layer_fused_cuda")
                launcher = _FusedLayerLauncher(self, meta, key[0], sm_scale)
                meta.launcher, meta.launcher_key = launcher, key
            if (rotary_dim, base) != launcher.rope_args:
                launcher.rope_checked = self._check_rope_args(rotary_dim, base)
                launcher.rope_args = (rotary_dim, base)
            rotary_dim = launcher.rope_checked
            if torch._C._cuda_getDevice() != self.device.index:
                with torch.cuda.device(self.device):
                    out = launcher.run(layer_idx, q, k, v, rotary_dim, float(base))
            else:
                out = launcher.run(layer_idx, q, k, v, rotary_dim, float(base))
        except Exception:
            self._ledger.transaction_failure_count += 1
            raise
        self._ledger.record_layer_write(state, layer_idx)
        return out, meta.public

    def commit_token(self, transaction):
        """Publish one token after every layer has been written."""
        state = self._require_open_transaction(transaction)
        if state.next_layer_idx != self.num_layers:
            raise RuntimeError("cannot commit token before all layers are written")
        view = replace(self._view(state), state="committed")
        self._ledger.commit_token(state)
        return view

    def abort_token(self, transaction):
        """Abort an open token and return the boundary blocks it reserved."""
        state = self._require_open_transaction(transaction)
        view = replace(self._view(state), state="aborted")
        self._ledger.abort_token(state)
        return view

    def transaction_view(self, transaction):
        state = self._require_transaction(transaction)
        if state.state != "open":
            raise RuntimeError(f"token transaction is already {state.state}")
        return self._view(state)

    def _view(self, state):
        pub = state.device_view.public
        return KVTokenTransactionView(
            transaction_id=state.transaction_id, cache_version=state.cache_version,
            request_ids=state.request_ids, positions=pub["positions"],
            physical_block_ids=pub["physical_block_ids"], block_offsets=pub["block_offsets"],
            block_tables=pub["block_tables"], effective_seq_lens=pub["effective_seq_lens"],
            next_layer_idx=state.next_layer_idx, state=state.state)

    def _require_transaction(self, transaction):
        if not isinstance(transaction, KVTokenTransactionView):
            raise TypeError("transaction must be a KVTokenTransactionView")
        return self._ledger.lookup_transaction(transaction.transaction_id,
                                               transaction.cache_version,
                                               transaction.request_ids)

    def _require_open_transaction(self, transaction):
        if not isinstance(transaction, KVTokenTransactionView):
            raise TypeError("transaction must be a KVTokenTransactionView")
        return self._ledger.require_open(transaction.transaction_id, transaction.cache_version,
                                         transaction.request_ids)

    def _prepare_transaction_layer_write(self, state, layer_idx, k, v):
        layer_idx = self._ledger.check_layer_for_write(state, layer_idx)
        _, ids, k, v = self._prepare_append_inputs(layer_idx, state.request_ids, k, v)
        if tuple(ids) != state.request_ids:
            raise RuntimeError("transaction request order changed unexpectedly")
        return layer_idx, k, v

    # --------------------------------------------------------------- views
    def block_tables(self, request_ids=None, max_blocks_per_seq=None, pad_value=-1):
        """Padded physical block ids ``[num_requests, max_blocks_per_seq]`` (int32)."""
        ids = self._normalize_active_request_ids(request_ids)
        rows = self._ledger.block_table_rows(ids, max_blocks_per_seq, pad_value)
        width = len(rows[0]) if rows else max(1, int(max_blocks_per_seq or 1))
        t = torch.tensor(rows, dtype=torch.int32) if rows else torch.full((0, width), int(pad_value),
                                                                          dtype=torch.int32)
        return t.to(self.device)

    def seq_lens_tensor(self, request_ids=None, device=None):
        ids = self._normalize_active_request_ids(request_ids)
        return torch.tensor([self._ledger.requests[r].seq_len for r in ids],
                            device=device if device is not None else self.device,
                            dtype=torch.int32)

    def to_dense(self, layer_idx=0, request_ids=None, max_seq_len=None):
        """Materialise ``[num_requests, max_seq_len, Hkv, D]`` dense K/V (debug)."""
        layer_idx = self._ledger.validate_layer_idx(layer_idx)
        ids = self._normalize_active_request_ids(request_ids)
        longest = max((self._ledger.requests[r].seq_len for r in ids), default=0)
        max_seq_len = int(max(1, longest) if max_seq_len is None else max_seq_len)
        if max_seq_len < longest:
            raise ValueError("max_seq_len is smaller than an existing request length")
        shape = (len(ids), max_seq_len, self.num_kv_heads, self.head_dim)
        k_dense = torch.zeros(shape, device=self.device, dtype=self.dtype)
        v_dense = torch.zeros_like(k_dense)
        for row, rid in enumerate(ids):
            st = self._ledger.requests[rid]
            if st.seq_len == 0:
                continue
            index = torch.tensor(st.block_ids, device=self.device, dtype=torch.long)
            kt = self.k_cache[layer_idx].index_select(0, index).permute(0, 2, 1, 3)
            vt = self.v_cache[layer_idx].index_select(0, index).permute(0, 2, 1, 3)
            k_dense[row, : st.seq_len] = kt.reshape(-1, self.num_kv_heads, self.head_dim)[: st.seq_len]
            v_dense[row, : st.seq_len] = vt.reshape(-1, self.num_kv_heads, self.head_dim)[: st.seq_len]
        return k_dense, v_dense, self.seq_lens_tensor(ids)

    def metrics(self):
        bytes_per_block = (self.num_layers * 2 * self.num_kv_heads * self.block_size *
                           self.head_dim * self.k_cache.element_size())
        return self._ledger.metrics(bytes_per_block)

    def validate_invariants(self):
        return self._ledger.validate_invariants()

    @property
    def num_free_blocks(self):
        return len(self._ledger.free)

    @property
    def num_used_blocks(self):
        return self.max_blocks - len(self._ledger.free)

    @property
    def state_version(self):
        return self._ledger.state_version

    @property
    def has_open_transaction(self):
        return self._ledger.open_transaction_id is not None

    # ------------------------------------------------------------- helpers
    def _require_cuda(self, what):
        if self.device.type != "cuda":
            raise ValueError(f"{what} requires a CUDA-resident PagedKVCache")

    def _check_rope_args(self, rotary_dim, base):
        if rotary_dim is None:
            rotary_dim = self.head_dim
        if isinstance(rotary_dim, bool) or not isinstance(rotary_dim, int):
            raise ValueError("rotary_dim must be an even integer")
        if rotary_dim <= 0 or rotary_dim > self.head_dim or rotary_dim % 2 != 0:
            raise ValueError("rotary_dim must be positive, even, and no larger than head_dim")
        base = float(base)
        if not math.isfinite(base) or base <= 0.0:
            raise ValueError("base must be a positive finite number")
        return rotary_dim

    def _prepare_append_inputs(self, layer_idx, request_ids, k, v):
        layer_idx = self._ledger.validate_layer_idx(layer_idx)
        ids = self._normalize_request_ids(request_ids)
        if not ids:
            raise ValueError("request_ids must be non-empty")
        if len(set(ids)) != len(ids):
            raise ValueError("request_ids must be unique within one append call")
        if k.dim() == 2 and len(ids) == 1:
            k = k.unsqueeze(0)
        if v.dim() == 2 and len(ids) == 1:
            v = v.unsqueeze(0)
        if k.dim() != 3 or v.dim() != 3:
            raise ValueError("k and v must have shape [num_requests, num_kv_heads, head_dim]")
        if k.shape != v.shape:
            raise ValueError("k and v must have the same shape")
        if k.shape != (len(ids), self.num_kv_heads, self.head_dim):
            raise ValueError("k and v shapes must match request count, num_kv_heads, and head_dim")
        if k.device != self.device or v.device != self.device:
            raise ValueError("k and v must be on the cache device")
        if k.dtype != self.dtype or v.dtype != self.dtype:
            raise ValueError("k and v must use the cache dtype")
        if not k.is_floating_point() or not v.is_floating_point():
            raise ValueError("k and v must be floating point tensors")
        return layer_idx, ids, k, v

    def _prepare_prefix_blocks(self, k_blocks, v_blocks):
        if not isinstance(k_blocks, torch.Tensor) or not isinstance(v_blocks, torch.Tensor):
            raise TypeError("k_blocks and v_blocks must be torch tensors")
        if k_blocks.dim() != 5 or v_blocks.dim() != 5:
            raise ValueError("prefix K/V must have shape "
                             "[num_layers, num_prefix_blocks, num_kv_heads, block_size, head_dim]")
        if k_blocks.shape != v_blocks.shape:
            raise ValueError("prefix k_blocks and v_blocks must have the same shape")
        tail = (self.num_kv_heads, self.block_size, self.head_dim)
        if k_blocks.shape[0] != self.num_layers or tuple(k_blocks.shape[2:]) != tail:
            raise ValueError("prefix K/V shape does not match the PagedKVCache layout")
        if k_blocks.shape[1] <= 0:
            raise ValueError("prefix must contain at least one full block")
        if k_blocks.device != self.device or v_blocks.device != self.device:
            raise ValueError("prefix K/V must be on the cache device")
        if k_blocks.dtype != self.dtype or v_blocks.dtype != self.dtype:
            raise ValueError("prefix K/V must use the cache dtype")
        return k_blocks, v_blocks

    def _normalize_request_ids(self, request_ids):
        if isinstance(request_ids, torch.Tensor):
            if request_ids.dim() == 0:
                ids = [int(request_ids.detach().cpu().item())]
            else:
                ids = [int(x) for x in request_ids.detach().cpu().reshape(-1).tolist()]
        elif isinstance(request_ids, (str, bytes)):
            ids = [request_ids]
        else:
            try:
                ids = list(request_ids)
            except TypeError:
                ids = [request_ids]
        for rid in ids:
            BlockLedger.check_request_id(rid)
        return ids

    def _normalize_active_request_ids(self, request_ids):
        ids = self._ledger.active_ids() if request_ids is None else self._normalize_request_ids(request_ids)
        for rid in ids:
            self._ledger.require_active(rid)
        return ids

    # reference-compatible private accessors used by callers/tests
    @property
    def _free_blocks(self):
        return self._ledger.free

    @property
    def _requests(self):
        return self._ledger.requests

    @property
    def _open_transaction_id(self):
        return self._ledger.open_transaction_id


Hashable  # re-export for annotations
