"""Physical-block ledger of the paged KV cache (pure Python, no tensors).

Holds every integer decision of ``PagedKVCache`` so that slot placement is
bit-exact with the reference and testable without a GPU.  Semantics follow
``flashdec/cache.py`` of cysong2025/flashdec:

* a FIFO free list of physical blocks; allocation pops the front, release
  pushes blocks back to the front in reverse order so they are reused first
  (:146, :1245-1255, :1318-1323);
* appending token ``pos`` of a request uses logical block ``pos // bs`` at
  offset ``pos % bs`` and allocates a new block exactly when
  ``pos % bs == 0`` (:470-478, :1226-1239);
* a multi-layer token transaction reserves one location per request for all
  layers, publishes ``seq_len + 1`` once at commit and returns its boundary
  blocks on abort (:438-515, :610-648);
* immutable shared prefixes: refcounted, LRU-evicted when inactive, attached
  only to empty requests (:192-276, :1365-1397).
Error types and messages match the reference.
"""

from __future__ import annotations

from collections import OrderedDict, deque
from dataclasses import dataclass, field
from typing import Hashable


@dataclass
class RequestState:
    status: str = "active"
    seq_len: int = 0
    block_ids: list = field(default_factory=list)
    transaction_id: int | None = None
    prefix_id: Hashable | None = None
    shared_block_count: int = 0


@dataclass
class PrefixState:
    block_ids: tuple
    active_refcount: int = 0


@dataclass
class TransactionState:
    transaction_id: int
    cache_version: int
    request_ids: tuple
    positions: tuple
    locations: tuple  # ((block_id, offset), ...)
    newly_allocated_by_request: dict
    allocation_order: tuple
    next_layer_idx: int = 0
    written_layers: set = field(default_factory=set)
    state: str = "open"
    device_view: object = None  # owned by PagedKVCache


@dataclass(frozen=True)
class TerminalTransaction:
    transaction_id: int
    cache_version: int
    request_ids: tuple
    state: str


class BlockLedger:
    ACTIVE = "active"
    FINISHED = "finished"
    CANCELLED = "cancelled"
    TERMINAL_HISTORY_LIMIT = 256

    def __init__(self, num_layers, block_size, max_blocks, prefix_cache_capacity_blocks=0):
        self.num_layers = int(num_layers)
        self.block_size = int(block_size)
        self.max_blocks = int(max_blocks)
        self.prefix_cache_capacity_blocks = int(prefix_cache_capacity_blocks)
        if self.prefix_cache_capacity_blocks < 0:
            raise ValueError("prefix_cache_capacity_blocks must be non-negative")
        if self.prefix_cache_capacity_blocks > self.max_blocks:
            raise ValueError("prefix_cache_capacity_blocks must not exceed max_blocks")
        self.free = deque(range(self.max_blocks))
        self.requests: dict = {}
        self.prefixes: OrderedDict = OrderedDict()
        self.ever_allocated: set = set()
        self.allocation_count = 0
        self.fresh_allocation_count = 0
        self.free_count = 0
        self.reuse_count = 0
        self.capacity_failure_count = 0
        self.state_version = 0
        self.next_transaction_id = 1
        self.open_transaction_id = None
        self.transactions: dict = {}
        self.terminal: OrderedDict = OrderedDict()
        self.terminal_limit = self.TERMINAL_HISTORY_LIMIT
        self.transaction_begin_count = 0
        self.transaction_commit_count = 0
        self.transaction_abort_count = 0
        self.transaction_layer_write_count = 0
        self.transaction_rollback_block_count = 0
        self.transaction_failure_count = 0
        self.prefix_registration_count = 0
        self.prefix_hit_count = 0
        self.prefix_miss_count = 0
        self.prefix_eviction_count = 0
        self.prefix_capacity_failure_count = 0

    # ------------------------------------------------------------- requests
    @staticmethod
    def check_request_id(request_id):
        try:
            hash(request_id)
        except TypeError as exc:
            raise ValueError("request ids must be hashable") from exc

    @staticmethod
    def check_prefix_id(prefix_id):
        if prefix_id is None:
            raise ValueError("prefix_id must not be None")
        try:
            hash(prefix_id)
        except TypeError as exc:
            raise ValueError("prefix ids must be hashable") from exc

    def add_request(self, request_id):
        if self.open_transaction_id is not None:
            raise RuntimeError("cannot add a request during an open token transaction")
        self.check_request_id(request_id)
        state = self.requests.get(request_id)
        if state is None:
            self.requests[request_id] = RequestState()
            self.state_version += 1
        elif state.status != self.ACTIVE:
            raise RuntimeError(
                f"request_id {request_id!r} is {state.status} and cannot be reactivated"
            )

    def require_request(self, request_id):
        state = self.requests.get(request_id)
        if state is None:
            raise KeyError(f"unknown request_id: {request_id!r}")
        return state

    def require_active(self, request_id):
        state = self.require_request(request_id)
        if state.status != self.ACTIVE:
            raise RuntimeError(f"request_id {request_id!r} is {state.status}, not active")
        return state

    def active_ids(self):
        return [rid for rid, st in self.requests.items() if st.status == self.ACTIVE]

    def close_request(self, request_id, terminal_status):
        if self.open_transaction_id is not None:
            raise RuntimeError("cannot close a request during an open token transaction")
        state = self.require_active(request_id)
        prefix = None
        if state.prefix_id is not None:
            prefix = self.prefixes.get(state.prefix_id)
            if prefix is None or prefix.active_refcount <= 0:
                raise RuntimeError("shared prefix reference accounting is inconsistent")
        released = tuple(state.block_ids[state.shared_block_count:])
        for block_id in reversed(released):
            self.free.appendleft(block_id)
        self.free_count += len(released)
        state.block_ids.clear()
        if prefix is not None:
            prefix.active_refcount -= 1
            self.prefixes.move_to_end(state.prefix_id)
        state.prefix_id = None
        state.shared_block_count = 0
        state.status = terminal_status
        self.state_version += 1
        return released

    # ----------------------------------------------------------- allocation
    def allocate_block(self):
        if not self.free:
            raise RuntimeError("PagedKVCache is out of physical blocks")
        block_id = self.free.popleft()
        self.allocation_count += 1
        if block_id in self.ever_allocated:
            self.reuse_count += 1
        else:
            self.ever_allocated.add(block_id)
            self.fresh_allocation_count += 1
        return block_id

    def preflight_append(self, ids):
        needed = 0
        for request_id in ids:
            state = self.requests.get(request_id)
            if state is not None and state.status != self.ACTIVE:
                raise RuntimeError(
                    f"request_id {request_id!r} is {state.status} and cannot accept append"
                )
            seq_len = 0 if state is None else state.seq_len
            if seq_len % self.block_size == 0:
                needed += 1
        if needed > len(self.free):
            self.capacity_failure_count += 1
            raise RuntimeError("PagedKVCache is out of physical blocks")

    def allocate_append_locations(self, ids):
        """Legacy single-layer append: reserve (block, offset) per request.
        Unknown ids become new requests (reference cache.py:1226-1239)."""
        locations = []
        for request_id in ids:
            state = self.requests.get(request_id)
            if state is None:
                state = RequestState()
                self.requests[request_id] = state
            pos = state.seq_len
            logical, offset = divmod(pos, self.block_size)
            if offset == 0:
                state.block_ids.append(self.allocate_block())
            locations.append((state.block_ids[logical], offset))
        return locations

    def advance_lengths(self, ids):
        for request_id in ids:
            self.requests[request_id].seq_len += 1
        self.state_version += 1

    def require_legacy_append_available(self):
        if self.num_layers != 1:
            raise RuntimeError("multi-layer cache writes require the token transaction API")
        if self.open_transaction_id is not None:
            raise RuntimeError("legacy append is not allowed during an open token transaction")

    def next_positions(self, ids):
        positions = []
        for request_id in ids:
            state = self.requests.get(request_id)
            if state is None:
                positions.append(0)
            elif state.status != self.ACTIVE:
                raise RuntimeError(
                    f"request_id {request_id!r} is {state.status} and cannot accept append"
                )
            elif state.transaction_id is not None:
                raise RuntimeError(f"request_id {request_id!r} belongs to an open token transaction")
            else:
                positions.append(state.seq_len)
        return positions

    # --------------------------------------------------------- transactions
    def begin_token(self, ids):
        if self.open_transaction_id is not None:
            raise RuntimeError("PagedKVCache already has an open token transaction")
        ids = tuple(ids)
        if not ids:
            raise ValueError("request_ids must be non-empty")
        if len(set(ids)) != len(ids):
            raise ValueError("request_ids must be unique within one token transaction")
        states = [self.require_active(rid) for rid in ids]
        if any(st.transaction_id is not None for st in states):
            raise RuntimeError("request already belongs to an open token transaction")
        needed = sum(st.seq_len % self.block_size == 0 for st in states)
        if needed > len(self.free):
            self.capacity_failure_count += 1
            self.transaction_failure_count += 1
            raise RuntimeError("PagedKVCache is out of physical blocks")

        transaction_id = self.next_transaction_id
        positions = tuple(st.seq_len for st in states)
        locations = []
        newly = {}
        order = []
        try:
            for rid, st, pos in zip(ids, states, positions):
                logical, offset = divmod(pos, self.block_size)
                if offset == 0:
                    block_id = self.allocate_block()
                    st.block_ids.append(block_id)
                    newly[rid] = block_id
                    order.append(block_id)
                locations.append((st.block_ids[logical], offset))
            self.validate_reserved_locations(ids, states, positions, locations)
            for st in states:
                st.transaction_id = transaction_id
        except Exception:
            for rid, block_id in newly.items():
                st = self.requests[rid]
                if st.block_ids and st.block_ids[-1] == block_id:
                    st.block_ids.pop()
                st.transaction_id = None
            for block_id in reversed(order):
                self.free.appendleft(block_id)
            self.transaction_failure_count += 1
            raise
        version = self.state_version + 1
        tx = TransactionState(transaction_id=transaction_id, cache_version=version,
                              request_ids=ids, positions=positions, locations=tuple(locations),
                              newly_allocated_by_request=newly, allocation_order=tuple(order))
        self.transactions[transaction_id] = tx
        self.open_transaction_id = transaction_id
        self.next_transaction_id += 1
        self.transaction_begin_count += 1
        self.state_version = version
        return tx

    def validate_reserved_locations(self, ids, states, positions, locations):
        """Prove the raw-kernel indices from host state (reference :1172-1208)."""
        if not len(ids) == len(states) == len(positions) == len(locations):
            raise RuntimeError("transaction location metadata has inconsistent rows")
        for rid, st, pos, (block_id, offset) in zip(ids, states, positions, locations):
            if pos < 0:
                raise RuntimeError("transaction position must be non-negative")
            if not 0 <= block_id < self.max_blocks:
                raise RuntimeError("transaction physical block id is out of range")
            if not 0 <= offset < self.block_size:
                raise RuntimeError("transaction block offset is out of range")
            if offset != pos % self.block_size:
                raise RuntimeError("transaction block offset does not match position")
            logical = pos // self.block_size
            if logical >= len(st.block_ids):
                raise RuntimeError("transaction logical block is not allocated")
            if st.block_ids[logical] != block_id:
                raise RuntimeError(f"transaction physical block does not match request {rid!r}")

    def lookup_transaction(self, transaction_id, cache_version, request_ids):
        state = self.transactions.get(transaction_id)
        if state is None:
            state = self.terminal.get(transaction_id)
        if state is None:
            raise RuntimeError("unknown token transaction")
        if cache_version != state.cache_version or tuple(request_ids) != state.request_ids:
            raise RuntimeError("stale or invalid token transaction handle")
        return state

    def require_open(self, transaction_id, cache_version, request_ids):
        state = self.lookup_transaction(transaction_id, cache_version, request_ids)
        if state.state != "open":
            raise RuntimeError(f"token transaction is already {state.state}")
        if self.open_transaction_id != state.transaction_id:
            raise RuntimeError("token transaction is not the current open transaction")
        return state

    def check_layer_for_write(self, state, layer_idx):
        layer_idx = self.validate_layer_idx(layer_idx)
        if layer_idx != state.next_layer_idx:
            raise RuntimeError(
                f"transaction requires layer {state.next_layer_idx}, got layer {layer_idx}"
            )
        return layer_idx

    def record_layer_write(self, state, layer_idx):
        state.written_layers.add(layer_idx)
        state.next_layer_idx += 1
        self.transaction_layer_write_count += 1

    def commit_token(self, state):
        if state.next_layer_idx != self.num_layers:
            raise RuntimeError("cannot commit token before all layers are written")
        for rid in state.request_ids:
            req = self.requests[rid]
            req.seq_len += 1
            req.transaction_id = None
        state.state = "committed"
        self.open_transaction_id = None
        self.transaction_commit_count += 1
        self.state_version += 1
        self.retire(state)

    def abort_token(self, state):
        for rid, block_id in state.newly_allocated_by_request.items():
            req = self.requests[rid]
            if not req.block_ids or req.block_ids[-1] != block_id:
                raise RuntimeError("transaction rollback block ownership is inconsistent")
        for rid in state.newly_allocated_by_request:
            self.requests[rid].block_ids.pop()
        for block_id in reversed(state.allocation_order):
            self.free.appendleft(block_id)
        for rid in state.request_ids:
            self.requests[rid].transaction_id = None
        state.state = "aborted"
        self.open_transaction_id = None
        self.transaction_abort_count += 1
        self.transaction_rollback_block_count += len(state.allocation_order)
        self.state_version += 1
        self.retire(state)

    def retire(self, state):
        retained = self.transactions.pop(state.transaction_id, None)
        if retained is not state:
            raise RuntimeError("token transaction retention state is inconsistent")
        state.device_view = None
        self.terminal[state.transaction_id] = TerminalTransaction(
            state.transaction_id, state.cache_version, state.request_ids, state.state)
        while len(self.terminal) > self.terminal_limit:
            self.terminal.popitem(last=False)

    def validate_layer_idx(self, layer_idx):
        layer_idx = int(layer_idx)
        if layer_idx < 0 or layer_idx >= self.num_layers:
            raise ValueError("layer_idx must be in [0, num_layers)")
        return layer_idx

    # -------------------------------------------------------------- prefixes
    def resident_prefix_blocks(self):
        return sum(len(p.block_ids) for p in self.prefixes.values())

    def prefix_eviction_plan(self, required):
        if required > self.prefix_cache_capacity_blocks:
            return None
        needed = max(0, self.resident_prefix_blocks() + required - self.prefix_cache_capacity_blocks,
                     required - len(self.free))
        if not needed:
            return ()
        released = 0
        victims = []
        for pid, prefix in self.prefixes.items():
            if prefix.active_refcount:
                continue
            victims.append(pid)
            released += len(prefix.block_ids)
            if released >= needed:
                return tuple(victims)
        return None

    def evict_prefix_entry(self, prefix_id):
        prefix = self.prefixes[prefix_id]
        if prefix.active_refcount:
            raise RuntimeError("cannot evict a prefix with active request references")
        del self.prefixes[prefix_id]
        for block_id in reversed(prefix.block_ids):
            self.free.appendleft(block_id)
        self.free_count += len(prefix.block_ids)
        self.prefix_eviction_count += 1
        return tuple(prefix.block_ids)

    def register_prefix(self, prefix_id, num_blocks):
        """Reserve ``num_blocks`` physical blocks for a new prefix; returns the
        block ids (the caller copies the data)."""
        if self.open_transaction_id is not None:
            raise RuntimeError("cannot register a prefix during an open token transaction")
        self.check_prefix_id(prefix_id)
        if prefix_id in self.prefixes:
            raise RuntimeError(f"prefix_id {prefix_id!r} is already registered")
        plan = self.prefix_eviction_plan(num_blocks)
        if plan is None:
            self.capacity_failure_count += 1
            self.prefix_capacity_failure_count += 1
            raise RuntimeError("PagedKVCache has insufficient evictable prefix capacity")
        for victim in plan:
            self.evict_prefix_entry(victim)
        return tuple(self.allocate_block() for _ in range(num_blocks))

    def publish_prefix(self, prefix_id, block_ids):
        self.prefixes[prefix_id] = PrefixState(block_ids=tuple(block_ids))
        self.prefix_registration_count += 1
        self.state_version += 1

    def attach_prefix(self, request_id, prefix_id):
        if self.open_transaction_id is not None:
            raise RuntimeError("cannot attach a prefix during an open token transaction")
        self.check_prefix_id(prefix_id)
        state = self.require_active(request_id)
        if state.transaction_id is not None:
            raise RuntimeError("cannot attach a prefix to a request in a token transaction")
        if state.seq_len or state.block_ids or state.prefix_id is not None:
            raise RuntimeError("shared prefixes can only attach to an empty active request")
        prefix = self.prefixes.get(prefix_id)
        if prefix is None:
            self.prefix_miss_count += 1
            raise KeyError(f"unknown prefix_id: {prefix_id!r}")
        state.block_ids.extend(prefix.block_ids)
        state.seq_len = len(prefix.block_ids) * self.block_size
        state.prefix_id = prefix_id
        state.shared_block_count = len(prefix.block_ids)
        prefix.active_refcount += 1
        self.prefixes.move_to_end(prefix_id)
        self.prefix_hit_count += 1
        self.state_version += 1
        return tuple(prefix.block_ids)

    def evict_prefix(self, prefix_id):
        if self.open_transaction_id is not None:
            raise RuntimeError("cannot evict a prefix during an open token transaction")
        self.check_prefix_id(prefix_id)
        prefix = self.prefixes.get(prefix_id)
        if prefix is None:
            raise KeyError(f"unknown prefix_id: {prefix_id!r}")
        if prefix.active_refcount:
            raise RuntimeError("cannot evict a prefix with active request references")
        released = self.evict_prefix_entry(prefix_id)
        self.state_version += 1
        return released

    def prefix_state(self, prefix_id):
        self.check_prefix_id(prefix_id)
        prefix = self.prefixes.get(prefix_id)
        if prefix is None:
            raise KeyError(f"unknown prefix_id: {prefix_id!r}")
        return {
            "prefix_id": prefix_id,
            "block_ids": tuple(prefix.block_ids),
            "num_blocks": len(prefix.block_ids),
            "token_count": len(prefix.block_ids) * self.block_size,
            "active_refcount": prefix.active_refcount,
        }

    # ---------------------------------------------------------------- views
    def block_table_rows(self, ids, max_blocks_per_seq=None, pad_value=-1):
        """Padded rows of physical block ids (list of lists)."""
        if max_blocks_per_seq is None:
            max_blocks_per_seq = max(1, max((len(self.requests[r].block_ids) for r in ids),
                                            default=0))
        max_blocks_per_seq = int(max_blocks_per_seq)
        if max_blocks_per_seq <= 0:
            raise ValueError("max_blocks_per_seq must be positive")
        rows = []
        for rid in ids:
            blocks = self.requests[rid].block_ids
            if len(blocks) > max_blocks_per_seq:
                raise ValueError("max_blocks_per_seq is smaller than a request's block count")
            rows.append(list(blocks) + [int(pad_value)] * (max_blocks_per_seq - len(blocks)))
        return rows

    def metrics(self, bytes_per_block):
        states = list(self.requests.values())
        active = [s for s in states if s.status == self.ACTIVE]
        used = self.max_blocks - len(self.free)
        resident_prefix = self.resident_prefix_blocks()
        active_prefix_refs = sum(p.active_refcount for p in self.prefixes.values())
        shared_prefix = sum(len(p.block_ids) for p in self.prefixes.values()
                            if p.active_refcount >= 2)
        saved_prefix = sum(max(0, p.active_refcount - 1) * len(p.block_ids)
                           for p in self.prefixes.values())
        open_tx = (self.transactions.get(self.open_transaction_id)
                   if self.open_transaction_id is not None else None)
        reserved_tx_blocks = len(open_tx.allocation_order) if open_tx is not None else 0
        reserved_tokens = used * self.block_size
        active_tokens = sum(s.seq_len for s in active)
        physical = resident_prefix * self.block_size + sum(
            max(0, s.seq_len - s.shared_block_count * self.block_size) for s in active)
        frag = reserved_tokens - physical
        lookups = self.prefix_hit_count + self.prefix_miss_count
        return {
            "max_blocks": self.max_blocks,
            "used_blocks": used,
            "free_blocks": len(self.free),
            "block_utilization": used / self.max_blocks,
            "active_tokens": active_tokens,
            "physical_data_tokens": physical,
            "reserved_tokens": reserved_tokens,
            "internal_fragmentation_tokens": frag,
            "internal_fragmentation_ratio": frag / reserved_tokens if reserved_tokens else 0.0,
            "allocation_count": self.allocation_count,
            "fresh_allocation_count": self.fresh_allocation_count,
            "free_count": self.free_count,
            "reuse_count": self.reuse_count,
            "capacity_failure_count": self.capacity_failure_count,
            "active_requests": sum(s.status == self.ACTIVE for s in states),
            "finished_requests": sum(s.status == self.FINISHED for s in states),
            "cancelled_requests": sum(s.status == self.CANCELLED for s in states),
            "transaction_begin_count": self.transaction_begin_count,
            "transaction_commit_count": self.transaction_commit_count,
            "transaction_abort_count": self.transaction_abort_count,
            "open_transaction_count": int(open_tx is not None),
            "retained_transaction_state_count": len(self.transactions),
            "terminal_transaction_history_count": len(self.terminal),
            "terminal_transaction_history_limit": self.terminal_limit,
            "pending_request_count": len(open_tx.request_ids) if open_tx is not None else 0,
            "reserved_transaction_blocks": reserved_tx_blocks,
            "transaction_layer_write_count": self.transaction_layer_write_count,
            "transaction_rollback_block_count": self.transaction_rollback_block_count,
            "transaction_failure_count": self.transaction_failure_count,
            "bytes_per_block": bytes_per_block,
            "allocated_kv_bytes": used * bytes_per_block,
            "reserved_transaction_bytes": reserved_tx_blocks * bytes_per_block,
            "prefix_cache_capacity_blocks": self.prefix_cache_capacity_blocks,
            "resident_prefix_count": len(self.prefixes),
            "resident_prefix_blocks": resident_prefix,
            "active_prefix_references": active_prefix_refs,
            "shared_prefix_blocks": shared_prefix,
            "saved_prefix_blocks": saved_prefix,
            "saved_prefix_bytes": saved_prefix * bytes_per_block,
            "prefix_registration_count": self.prefix_registration_count,
            "prefix_hit_count": self.prefix_hit_count,
            "prefix_miss_count": self.prefix_miss_count,
            "prefix_hit_ratio": self.prefix_hit_count / lookups if lookups else 0.0,
            "prefix_eviction_count": self.prefix_eviction_count,
            "prefix_capacity_failure_count": self.prefix_capacity_failure_count,
        }

    def validate_invariants(self):
        """Raise RuntimeError if ownership and the free list diverge
        (reference cache.py:805-943)."""
        free = list(self.free)
        if len(free) != len(set(free)):
            raise RuntimeError("PagedKVCache free list contains duplicate blocks")
        prefix_blocks = []
        expected_refs = {pid: 0 for pid in self.prefixes}
        for prefix in self.prefixes.values():
            if not prefix.block_ids:
                raise RuntimeError("resident prefix must own at least one block")
            if prefix.active_refcount < 0:
                raise RuntimeError("prefix active_refcount must be non-negative")
            prefix_blocks.extend(prefix.block_ids)
        if len(prefix_blocks) != len(set(prefix_blocks)):
            raise RuntimeError("a physical block belongs to multiple prefixes")
        if len(prefix_blocks) > self.prefix_cache_capacity_blocks:
            raise RuntimeError("resident prefixes exceed configured prefix capacity")
        private = []
        for st in self.requests.values():
            if st.status == self.ACTIVE:
                pending = int(st.transaction_id is not None)
                expected = (st.seq_len + pending + self.block_size - 1) // self.block_size
                if len(st.block_ids) != expected:
                    raise RuntimeError("active request block count does not match seq_len")
                if st.prefix_id is None:
                    if st.shared_block_count:
                        raise RuntimeError("request without prefix has shared blocks")
                else:
                    prefix = self.prefixes.get(st.prefix_id)
                    if prefix is None:
                        raise RuntimeError("request references a non-resident prefix")
                    if st.shared_block_count != len(prefix.block_ids):
                        raise RuntimeError("request shared block count does not match prefix")
                    if tuple(st.block_ids[: st.shared_block_count]) != prefix.block_ids:
                        raise RuntimeError("request shared block ids do not match prefix")
                    if st.seq_len < st.shared_block_count * self.block_size:
                        raise RuntimeError("request seq_len is shorter than its shared prefix")
                    expected_refs[st.prefix_id] += 1
                private.extend(st.block_ids[st.shared_block_count:])
            else:
                if st.block_ids:
                    raise RuntimeError("terminal request still owns physical blocks")
                if st.transaction_id is not None:
                    raise RuntimeError("terminal request belongs to a token transaction")
                if st.prefix_id is not None or st.shared_block_count:
                    raise RuntimeError("terminal request still references a shared prefix")
        for pid, prefix in self.prefixes.items():
            if prefix.active_refcount != expected_refs[pid]:
                raise RuntimeError("prefix active_refcount does not match attached requests")
        if len(private) != len(set(private)):
            raise RuntimeError("a private physical block is owned by multiple requests")
        if set(private) & set(prefix_blocks):
            raise RuntimeError("a physical block is both private and prefix-owned")
        owned = prefix_blocks + private
        if set(owned) & set(free):
            raise RuntimeError("a physical block is both owned and free")
        if set(owned) | set(free) != set(range(self.max_blocks)):
            raise RuntimeError("physical block accounting does not cover the cache")
        if len(self.transactions) > 1:
            raise RuntimeError("PagedKVCache retains more than one transaction state")
        if any(t.state != "open" for t in self.transactions.values()):
            raise RuntimeError("terminal transaction retained device-backed state")
        if len(self.terminal) > self.terminal_limit:
            raise RuntimeError("terminal transaction history exceeds its limit")
        if set(self.transactions) & set(self.terminal):
            raise RuntimeError("transaction appears in both open and terminal state")
        if any(t.state not in {"committed", "aborted"} for t in self.terminal.values()):
            raise RuntimeError("terminal transaction history contains an open state")
        ids = tuple(self.terminal)
        if any(tid != t.transaction_id for tid, t in self.terminal.items()):
            raise RuntimeError("terminal transaction history key does not match its state")
        if any(tid <= 0 or tid >= self.next_transaction_id for tid in ids):
            raise RuntimeError("terminal transaction history contains an invalid id")
        if any(t.cache_version <= 0 or t.cache_version > self.state_version
               for t in self.terminal.values()):
            raise RuntimeError("terminal transaction history contains an invalid version")
        if ids != tuple(sorted(ids)):
            raise RuntimeError("terminal transaction history is not ordered by id")
        open_states = list(self.transactions.values())
        if self.open_transaction_id is None:
            if open_states:
                raise RuntimeError("open transaction is missing from cache state")
            if any(s.transaction_id is not None for s in self.requests.values()):
                raise RuntimeError("request has an in-flight marker without an open transaction")
        else:
            if len(open_states) != 1:
                raise RuntimeError("PagedKVCache must have exactly one open transaction")
            tx = open_states[0]
            if tx.transaction_id != self.open_transaction_id:
                raise RuntimeError("open transaction id does not match cache state")
            if tx.written_layers != set(range(tx.next_layer_idx)):
                raise RuntimeError("transaction written layers are not sequential")
            if not 0 <= tx.next_layer_idx <= self.num_layers:
                raise RuntimeError("transaction next layer is out of range")
            for rid, pos, loc in zip(tx.request_ids, tx.positions, tx.locations):
                req = self.require_active(rid)
                if req.transaction_id != tx.transaction_id:
                    raise RuntimeError("request transaction marker does not match")
                if pos != req.seq_len:
                    raise RuntimeError("transaction position is not the committed seq_len")
                if loc != (req.block_ids[pos // self.block_size], pos % self.block_size):
                    raise RuntimeError("transaction physical location does not match ownership")
        return True
