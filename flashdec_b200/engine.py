"""Transactional decode engine over the B200 kernels.

Drop-in for ``flashdec/engine.py`` (cysong2025/flashdec) for the decode data
path: the request lifecycle (add / admit / finish / cancel), shared prefixes,
and the multi-layer token transaction

    tx  = engine.begin_step(ids)                       # engine.py:594-642
    res = engine.step_layer(tx, layer, q, k, v, ...)   # engine.py:644-724
    out = engine.commit_step(tx)                       # engine.py:726-747
          engine.abort_step(tx)                        # engine.py:749-752

plus the single-layer ``step`` wrapper (engine.py:754-871), ``metrics`` and
``validate_invariants``, with the reference's dataclasses, state names,
validation order and error messages.

With ``append_backend='fused_cuda'`` each layer is ONE launch on the
caller's stream: ``fd_paged_decode`` with its fused-append and RoPE fields,
which rotates q and the new K row, stores K/V at the slots reserved by
``begin_step`` and attends over the transaction's block tables and effective
lengths.  The other append backends run ``fd_rope_kv_append`` and then
``fd_paged_decode`` (two launches; same arithmetic).  The transaction
metadata is uploaded once per token by the cache and read by every layer;
nothing in a layer synchronises with the device.

Differences from the reference, by design:

* ``decode_backend`` is ``'cuda'`` (``'triton'`` is accepted as an alias so
  reference call sites keep working).  ``'reference'`` -- the reference's CPU
  semantic oracle -- is not part of this package and is rejected.
* All append backends run native kernels (see :mod:`flashdec_b200.rope`).
* Scheduler-managed mode (``submit_request``, ``scheduling_snapshot``,
  ``apply_scheduler_decision``, ``prefill_request[_layers]``; engine.py:200-
  573 with flashdec/scheduler.py) is an admission policy outside the decode
  data path; those methods raise ``NotImplementedError``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Hashable

import torch

PROFILE_RANGE_PREFLIGHT = "flashdec::engine_preflight"
PROFILE_RANGE_APPEND = "flashdec::rope_kv_append"
PROFILE_RANGE_DECODE = "flashdec::paged_decode"


@dataclass(frozen=True)
class AdmissionResult:
    """State transition result for a request submitted to the engine."""

    request_id: Hashable
    status: str


@dataclass(frozen=True)
class DecodeStepResult:
    """One decode-step result, or an explicit backpressure response."""

    status: str
    request_ids: tuple
    output: Any | None
    positions: Any | None
    block_tables: Any | None
    seq_lens: Any | None
    needed_new_blocks: int
    free_blocks: int
    reason: str | None = None


@dataclass(frozen=True)
class DecodeStepTransaction:
    """Stable handle for one open multi-layer token transaction."""

    transaction_id: int
    engine_version: int
    request_ids: tuple
    positions: Any
    physical_block_ids: Any
    block_offsets: Any
    block_tables: Any
    effective_seq_lens: Any


@dataclass(frozen=True)
class DecodeLayerResult:
    """Output of one layer inside an open token transaction."""

    transaction_id: int
    layer_idx: int
    request_ids: tuple
    output: Any
    positions: Any
    block_tables: Any
    effective_seq_lens: Any


class _OpenStep:
    """Engine-side state of the open transaction."""

    __slots__ = ("handle", "cache_tx", "needed_new_blocks", "next_layer_idx", "last_output",
                 "state")

    def __init__(self, handle, cache_tx, needed_new_blocks):
        self.handle = handle
        self.cache_tx = cache_tx
        self.needed_new_blocks = needed_new_blocks
        self.next_layer_idx = 0
        self.last_output = None
        self.state = "open"


_SCHEDULER_MSG = ("scheduler-managed mode is outside flashdec_b200's decode data path; "
                  "use add_request/admit and begin_step/step_layer/commit_step")


class DecodeEngine:
    """Request lifecycle + RoPE/KV append + paged decode (see module doc)."""

    WAITING = "waiting"
    ACTIVE = "active"
    FINISHED = "finished"
    CANCELLED = "cancelled"
    REJECTED = "rejected"

    STEP_OK = "ok"
    STEP_BACKPRESSURE = "backpressure"

    _APPEND_BACKENDS = ("torch", "cuda", "fused_cuda")
    _DECODE_BACKENDS = ("cuda", "triton")

    def __init__(self, cache, append_backend="torch", decode_backend="cuda", sm_scale=None,
                 num_warps=2, num_stages=None, profile_ranges=False):
        from .cache import PagedKVCache

        if not isinstance(cache, PagedKVCache):
            raise TypeError("cache must be a PagedKVCache")
        if append_backend not in self._APPEND_BACKENDS:
            raise ValueError("append_backend must be 'torch', 'cuda', or 'fused_cuda'")
        if decode_backend == "reference":
            raise ValueError("decode_backend='reference' (the CPU semantic oracle) is not part "
                             "of flashdec_b200; use 'cuda'")
        if decode_backend not in self._DECODE_BACKENDS:
            raise ValueError("decode_backend must be 'cuda' or 'triton'")
        if not isinstance(profile_ranges, bool):
            raise ValueError("profile_ranges must be a bool")
        self.cache = cache
        self.append_backend = append_backend
        self.decode_backend = decode_backend
        self.sm_scale = sm_scale
        self.num_warps = num_warps
        self.num_stages = num_stages
        self.profile_ranges = profile_ranges
        self._range = torch.profiler.record_function if profile_ranges else None
        self._statuses: dict = {}
        self._completed_step_count = 0
        self._appended_token_count = 0
        self._backpressure_count = 0
        self._state_version = 0
        self._open: _OpenStep | None = None
        self._transaction_layer_step_count = 0
        self._transaction_abort_count = 0

    # ------------------------------------------------------------ prefixes
    def register_prefix(self, prefix_id, k_blocks, v_blocks):
        """Register shared full blocks before any request enters the engine."""
        self._require_no_open_step("register a shared prefix")
        if self._statuses:
            raise RuntimeError("shared prefixes must be registered before request submission")
        m = self.cache.metrics()
        if any(m[name] for name in ("active_requests", "finished_requests",
                                    "cancelled_requests")):
            raise RuntimeError("shared prefix registration requires an empty PagedKVCache")
        return self.cache.register_prefix(prefix_id, k_blocks, v_blocks)

    def evict_prefix(self, prefix_id):
        """Evict one inactive prefix once every request lifecycle is resolved."""
        self._require_no_open_step("evict a shared prefix")
        if any(s in (self.WAITING, self.ACTIVE) for s in self._statuses.values()):
            raise RuntimeError("shared prefixes can only be evicted after all requests are "
                               "resolved")
        released = self.cache.evict_prefix(prefix_id)
        self._bump_state_version()
        return released

    # ----------------------------------------------------------- lifecycle
    def add_request(self, request_id):
        """Submit a request in ``waiting`` state (no KV memory is reserved)."""
        self._require_no_open_step("submit a request")
        self._check_request_id(request_id)
        if request_id in self._statuses:
            raise RuntimeError(f"request_id {request_id!r} already exists in the DecodeEngine")
        self._statuses[request_id] = self.WAITING
        self._bump_state_version()
        return AdmissionResult(request_id=request_id, status=self.WAITING)

    def admit(self, request_ids=None):
        """Move waiting requests to active (blocks are reserved per token)."""
        self._require_no_open_step("admit requests")
        ids = self._normalize_waiting_ids(request_ids)
        for rid in ids:
            self.cache.add_request(rid)
            self._statuses[rid] = self.ACTIVE
        self._bump_state_version()
        return tuple(AdmissionResult(request_id=rid, status=self.ACTIVE) for rid in ids)

    def submit_request(self, spec):
        raise NotImplementedError(_SCHEDULER_MSG)

    def scheduling_snapshot(self, logical_step, **kwargs):
        raise NotImplementedError(_SCHEDULER_MSG)

    def apply_scheduler_decision(self, decision, *, scheduler, snapshot):
        raise NotImplementedError(_SCHEDULER_MSG)

    def prefill_request(self, request_id, k, v, layer_idx=0):
        raise NotImplementedError(_SCHEDULER_MSG)

    def prefill_request_layers(self, request_id, k_layers, v_layers):
        raise NotImplementedError(_SCHEDULER_MSG)

    @property
    def state_version(self):
        """Monotonic engine lifecycle/sequence version."""
        return self._state_version

    def active_request_ids(self):
        """Active request ids in submission order."""
        return tuple(r for r, s in self._statuses.items() if s == self.ACTIVE)

    def request_state(self, request_id):
        status = self._require_known_request(request_id)
        result = {"request_id": request_id, "status": status}
        if status not in (self.WAITING, self.REJECTED):
            result["cache"] = self.cache.request_state(request_id)
        return result

    def finish_request(self, request_id):
        """Finish an active request and release its blocks."""
        self._require_no_open_step("finish a request")
        self._require_status(request_id, self.ACTIVE)
        released = self.cache.finish_request(request_id)
        self._statuses[request_id] = self.FINISHED
        self._bump_state_version()
        return released

    def cancel_request(self, request_id):
        """Cancel an active request and release its blocks."""
        self._require_no_open_step("cancel a request")
        self._require_status(request_id, self.ACTIVE)
        released = self.cache.cancel_request(request_id)
        self._statuses[request_id] = self.CANCELLED
        self._bump_state_version()
        return released

    # -------------------------------------------------------- transactions
    def begin_step(self, request_ids=None):
        """Reserve one token location per request for every layer."""
        self._require_no_open_step("begin another decode step")
        if self.append_backend not in ("torch", "fused_cuda"):
            raise RuntimeError(
                "multi-layer transactions require append_backend='torch' or 'fused_cuda'")
        ids = self._normalize_active_ids(request_ids)
        needed = self._needed_new_blocks(ids)
        if needed > self.cache.num_free_blocks:
            self._backpressure_count += 1
            raise RuntimeError("insufficient physical blocks to begin decode step")
        ctx = self.cache.begin_token(ids)
        # The view's tensors are already this token's public copies (the
        # kernels read the cache's internal buffers), so the handle takes them
        # as they are: one device copy of the metadata per token.
        handle = DecodeStepTransaction(
            transaction_id=ctx.transaction_id, engine_version=self._state_version + 1,
            request_ids=tuple(ids), positions=ctx.positions,
            physical_block_ids=ctx.physical_block_ids, block_offsets=ctx.block_offsets,
            block_tables=ctx.block_tables, effective_seq_lens=ctx.effective_seq_lens)
        self._bump_state_version()
        self._open = _OpenStep(handle, ctx, needed)
        return handle

    def step_layer(self, transaction, layer_idx, q, k, v, *, rotary_dim=None, base=10_000.0):
        """RoPE + K/V write and paged decode of one layer of the open token.

        Any exception aborts the whole token: committed lengths and block
        ownership stay as they were before ``begin_step``."""
        st = self._require_open_step(transaction)
        try:
            layer_idx = int(layer_idx)
            if layer_idx != st.next_layer_idx:
                raise RuntimeError(f"decode transaction requires layer {st.next_layer_idx}, "
                                   f"got layer {layer_idx}")
            self._validate_step_inputs(st.handle.request_ids, q, k, v)
            if k.dim() == 2:
                k = k.unsqueeze(0)
            if v.dim() == 2:
                v = v.unsqueeze(0)
            if self.append_backend == "fused_cuda" and self._range is None:
                # one prepared launch per layer: RoPE + K/V store + decode
                # (same arithmetic as the checked two-launch path below)
                out, pub = self.cache._fused_layer_step(st.cache_tx, layer_idx, q, k, v,
                                                        rotary_dim, base, self.sm_scale)
                st.next_layer_idx += 1
                st.last_output = out
                self._transaction_layer_step_count += 1
                return DecodeLayerResult(
                    transaction_id=st.handle.transaction_id, layer_idx=layer_idx,
                    request_ids=st.handle.request_ids, output=out,
                    positions=pub["positions"], block_tables=pub["block_tables"],
                    effective_seq_lens=pub["effective_seq_lens"])
            if self._range is None:
                q_rot, view = self._write_layer(st, layer_idx, q, k, v, rotary_dim, base)
                out = self._decode(q_rot, view.block_tables, view.effective_seq_lens, layer_idx)
            else:
                with self._range(PROFILE_RANGE_APPEND):
                    q_rot, view = self._write_layer(st, layer_idx, q, k, v, rotary_dim, base)
                with self._range(PROFILE_RANGE_DECODE):
                    out = self._decode(q_rot, view.block_tables, view.effective_seq_lens,
                                       layer_idx)
        except Exception:
            self._abort_open(st)
            raise
        st.next_layer_idx += 1
        st.last_output = out
        self._transaction_layer_step_count += 1
        return DecodeLayerResult(transaction_id=st.handle.transaction_id, layer_idx=layer_idx,
                                 request_ids=st.handle.request_ids, output=out,
                                 positions=view.positions, block_tables=view.block_tables,
                                 effective_seq_lens=view.effective_seq_lens)

    def commit_step(self, transaction):
        """Publish the token once every layer has run."""
        st = self._require_open_step(transaction)
        if st.next_layer_idx != self.cache.num_layers:
            raise RuntimeError("cannot commit decode step before all layers are complete")
        committed = self.cache.commit_token(st.cache_tx)
        st.state = "committed"
        self._open = None
        self._completed_step_count += 1
        self._appended_token_count += len(st.handle.request_ids)
        self._bump_state_version()
        return DecodeStepResult(
            status=self.STEP_OK, request_ids=st.handle.request_ids, output=st.last_output,
            positions=committed.positions, block_tables=committed.block_tables,
            # the committed lengths are the transaction's effective lengths
            # (position + 1); copying the device tensor keeps the host from
            # waiting for the step's kernels (a host-built tensor would be a
            # blocking upload behind them)
            seq_lens=st.handle.effective_seq_lens.clone(),
            needed_new_blocks=st.needed_new_blocks, free_blocks=self.cache.num_free_blocks)

    def abort_step(self, transaction):
        """Abort the open token transaction explicitly."""
        return self._abort_open(self._require_open_step(transaction))

    def step(self, q, k, v, request_ids=None, layer_idx=0, rotary_dim=None, base=10_000.0):
        """One append -> paged decode step on a single-layer cache.

        Capacity pressure returns ``status='backpressure'`` and changes no
        state; row order of ``request_ids`` is kept in every result tensor."""
        self._require_no_open_step("run the single-layer step wrapper")
        if self.cache.num_layers != 1:
            raise RuntimeError("multi-layer caches require begin_step/step_layer/commit_step")
        ids = self._normalize_active_ids(request_ids)
        self._validate_step_inputs(ids, q, k, v)
        needed = self._needed_new_blocks(ids)
        if needed > self.cache.num_free_blocks:
            self._backpressure_count += 1
            return DecodeStepResult(status=self.STEP_BACKPRESSURE, request_ids=ids, output=None,
                                    positions=None, block_tables=None, seq_lens=None,
                                    needed_new_blocks=needed,
                                    free_blocks=self.cache.num_free_blocks,
                                    reason="insufficient_physical_blocks")
        if self.append_backend == "torch":
            if int(layer_idx) != 0:
                raise ValueError("single-layer step requires layer_idx=0")
            tx = self.begin_step(ids)
            self.step_layer(tx, 0, q, k, v, rotary_dim=rotary_dim, base=base)
            return self.commit_step(tx)

        from .rope import rope_paged_kv_append

        res = rope_paged_kv_append(self.cache, layer_idx, ids, q, k, v, rotary_dim=rotary_dim,
                                   base=base, append_backend=self.append_backend)
        out = self._decode(res.q, res.block_tables, res.seq_lens)
        self._completed_step_count += 1
        self._appended_token_count += len(ids)
        self._bump_state_version()
        return DecodeStepResult(status=self.STEP_OK, request_ids=ids, output=out,
                                positions=res.positions, block_tables=res.block_tables,
                                seq_lens=res.seq_lens, needed_new_blocks=needed,
                                free_blocks=self.cache.num_free_blocks)

    # ------------------------------------------------------------- metrics
    def metrics(self):
        """Engine counters together with the cache metrics."""
        counts = {s: 0 for s in (self.WAITING, self.ACTIVE, self.FINISHED, self.CANCELLED,
                                 self.REJECTED)}
        for s in self._statuses.values():
            counts[s] += 1
        return {
            "waiting_requests": counts[self.WAITING],
            "active_requests": counts[self.ACTIVE],
            "finished_requests": counts[self.FINISHED],
            "cancelled_requests": counts[self.CANCELLED],
            "rejected_requests": counts[self.REJECTED],
            "completed_step_count": self._completed_step_count,
            "appended_token_count": self._appended_token_count,
            "backpressure_count": self._backpressure_count,
            "state_version": self._state_version,
            "cache_state_version": self.cache.state_version,
            "scheduler_managed": False,
            "committed_blocks": 0,
            "committed_but_unallocated_blocks": 0,
            "stale_decision_count": 0,
            "applied_decision_count": 0,
            "open_step_transaction_count": int(self._open is not None),
            "transaction_layer_step_count": self._transaction_layer_step_count,
            "transaction_abort_count": self._transaction_abort_count,
            "append_backend": self.append_backend,
            "decode_backend": self.decode_backend,
            "cache": self.cache.metrics(),
        }

    def validate_invariants(self):
        """Check that engine lifecycle state agrees with cache ownership."""
        self.cache.validate_invariants()
        if self._open is None:
            if self.cache.has_open_transaction:
                raise RuntimeError("cache has an open transaction not owned by DecodeEngine")
        else:
            if not self.cache.has_open_transaction:
                raise RuntimeError("Engine transaction is open but cache transaction is not")
            view = self.cache.transaction_view(self._open.cache_tx)
            if view.request_ids != self._open.handle.request_ids:
                raise RuntimeError("Engine/cache transaction request rows diverged")
            if view.next_layer_idx != self._open.next_layer_idx:
                raise RuntimeError("Engine/cache transaction layer progress diverged")
        for rid, status in self._statuses.items():
            if status in (self.WAITING, self.REJECTED):
                try:
                    self.cache.request_state(rid)
                except KeyError:
                    continue
                raise RuntimeError("waiting request unexpectedly exists in PagedKVCache")
            if self.cache.request_state(rid)["status"] != status:
                raise RuntimeError("DecodeEngine and PagedKVCache request status diverged")
        return True

    # ------------------------------------------------------------- helpers
    def _write_layer(self, st, layer_idx, q, k, v, rotary_dim, base):
        if self.append_backend == "fused_cuda":
            return self.cache.write_token_layer_fused_cuda(st.cache_tx, layer_idx, q, k, v,
                                                           rotary_dim=rotary_dim, base=base)
        from .rope import apply_rope

        ctx = self.cache.transaction_view(st.cache_tx)
        q_rot = apply_rope(q, ctx.positions, rotary_dim=rotary_dim, base=base)
        k_rot = apply_rope(k, ctx.positions, rotary_dim=rotary_dim, base=base)
        return q_rot, self.cache.write_token_layer(st.cache_tx, layer_idx, k_rot, v)

    def _decode(self, q, block_tables, seq_lens, layer_idx=0):
        layer_idx = int(layer_idx)
        if layer_idx < 0 or layer_idx >= self.cache.num_layers:
            raise ValueError("layer_idx must be in [0, num_layers)")
        from .kernels.paged_decode import paged_decode_attention

        return paged_decode_attention(q, self.cache.k_cache[layer_idx],
                                      self.cache.v_cache[layer_idx], block_tables, seq_lens,
                                      sm_scale=self.sm_scale, block_size=self.cache.block_size,
                                      num_warps=self.num_warps, num_stages=self.num_stages)

    def _abort_open(self, st):
        if self._open is not st or st.state != "open":
            raise RuntimeError("decode step transaction is not open")
        aborted = self.cache.abort_token(st.cache_tx)
        st.state = "aborted"
        self._open = None
        self._transaction_abort_count += 1
        self._bump_state_version()
        return aborted

    def _bump_state_version(self):
        self._state_version += 1

    def _require_no_open_step(self, action):
        if self._open is not None:
            raise RuntimeError(f"cannot {action} during an open decode step transaction")

    def _require_open_step(self, transaction):
        if not isinstance(transaction, DecodeStepTransaction):
            raise TypeError("transaction must be a DecodeStepTransaction")
        st = self._open
        if st is None:
            raise RuntimeError("DecodeEngine has no open decode step transaction")
        h = st.handle
        if (transaction.transaction_id != h.transaction_id
                or transaction.engine_version != h.engine_version
                or transaction.request_ids != h.request_ids):
            raise RuntimeError("stale or invalid DecodeEngine transaction handle")
        if st.state != "open":
            raise RuntimeError(f"decode step transaction is already {st.state}")
        return st

    def _validate_step_inputs(self, ids, q, k, v):
        if not all(isinstance(t, torch.Tensor) for t in (q, k, v)):
            raise TypeError("q, k, and v must be torch tensors")
        if q.dim() != 3:
            raise ValueError("q must have shape [num_requests, num_q_heads, head_dim]")
        if k.dim() == 2 and len(ids) == 1:
            k = k.unsqueeze(0)
        if v.dim() == 2 and len(ids) == 1:
            v = v.unsqueeze(0)
        c = self.cache
        expected = (len(ids), c.num_kv_heads, c.head_dim)
        if q.shape[0] != len(ids) or q.shape[1] <= 0 or q.shape[2] != c.head_dim:
            raise ValueError("q shape must match active request count and cache head_dim")
        if k.shape != expected or v.shape != expected:
            raise ValueError("k and v shapes must match active request count and cache "
                             "dimensions")
        if q.device != c.device or k.device != c.device or v.device != c.device:
            raise ValueError("q, k, and v must be on the cache device")
        if q.dtype != c.dtype or k.dtype != c.dtype or v.dtype != c.dtype:
            raise ValueError("q, k, and v must use the cache dtype")

    def _needed_new_blocks(self, ids):
        bs = self.cache.block_size
        ledger = self.cache._ledger
        return sum(ledger.require_request(r).seq_len % bs == 0 for r in ids)

    def _normalize_waiting_ids(self, request_ids):
        if request_ids is None:
            ids = tuple(r for r, s in self._statuses.items() if s == self.WAITING)
        else:
            ids = self._normalize_ids(request_ids)
        if not ids:
            raise ValueError("at least one waiting request is required for admission")
        for rid in ids:
            self._require_status(rid, self.WAITING)
        return ids

    def _normalize_active_ids(self, request_ids):
        ids = self.active_request_ids() if request_ids is None else self._normalize_ids(
            request_ids)
        if not ids:
            raise ValueError("at least one active request is required for a decode step")
        for rid in ids:
            self._require_status(rid, self.ACTIVE)
        return ids

    def _normalize_ids(self, request_ids):
        if isinstance(request_ids, (str, bytes)):
            ids = (request_ids,)
        else:
            try:
                ids = tuple(request_ids)
            except TypeError:
                ids = (request_ids,)
        for rid in ids:
            self._check_request_id(rid)
        if len(set(ids)) != len(ids):
            raise ValueError("request_ids must be unique")
        return ids

    @staticmethod
    def _check_request_id(request_id):
        try:
            hash(request_id)
        except TypeError as exc:
            raise ValueError("request ids must be hashable") from exc

    def _require_known_request(self, request_id):
        self._check_request_id(request_id)
        if request_id not in self._statuses:
            raise KeyError(f"unknown request_id: {request_id!r}")
        return self._statuses[request_id]

    def _require_status(self, request_id, expected):
        status = self._require_known_request(request_id)
        if status != expected:
            raise RuntimeError(f"request_id {request_id!r} is {status}, expected {expected}")
