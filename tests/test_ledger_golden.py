"""BlockLedger (the integer core of PagedKVCache) against the reference trace.

``tests/golden/ledger_golden.json`` was produced by running the reference's
own ``flashdec.cache.PagedKVCache`` through the script in
``tests/golden/make_golden.py::ledger_fixture``.  The same script is replayed
here on the ledger alone (no tensors, no GPU): every free list, block table,
slot (block id, offset), position, effective length, state version and
metric must be identical (bit-exact integer parity).
"""

from __future__ import annotations

import json

import pytest

from flashdec_b200.ledger import BlockLedger
from tests.golden.make_golden import LEDGER_METRICS

BYTES_PER_BLOCK = 2 * 2 * 1 * 8 * 2 * 4  # layers * (K,V) * heads * bs * dim * fp32


class _Replay:
    """Drives BlockLedger through the steps of ``ledger_fixture``."""

    def __init__(self):
        self.ledger = BlockLedger(num_layers=2, block_size=8, max_blocks=24,
                                  prefix_cache_capacity_blocks=6)
        self.log = []

    def active(self):
        return [r for r, st in self.ledger.requests.items() if st.status == "active"]

    def snap(self, tag, extra=None):
        led = self.ledger
        ids = self.active()
        rec = {
            "tag": tag,
            "free": list(led.free),
            "state_version": led.state_version,
            "block_ids": {str(r): list(led.requests[r].block_ids) for r in ids},
            "seq_lens": {str(r): led.requests[r].seq_len for r in ids},
        }
        if ids:
            rec["active"] = [str(r) for r in ids]
            rec["block_tables"] = [list(row) for row in led.block_table_rows(ids)]
        m = led.metrics(BYTES_PER_BLOCK)
        rec["metrics"] = {k: m[k] for k in LEDGER_METRICS}
        if extra:
            rec.update(extra)
        self.log.append(rec)

    def register_prefix(self, pid, nblocks):
        block_ids = self.ledger.register_prefix(pid, nblocks)
        self.ledger.publish_prefix(pid, block_ids)

    def run(self):
        led = self.ledger
        self.register_prefix("sys", 2)
        self.snap("register_prefix")
        for rid in ("a", "b", "c"):
            led.add_request(rid)
        led.attach_prefix("c", "sys")
        self.snap("add_requests")
        for step in range(30):
            ids = self.active()
            if step % 3 == 1:
                ids = list(reversed(ids))
            tx = led.begin_token(tuple(ids))
            rows = led.block_table_rows(tuple(ids))
            extra = {
                "ids": [str(r) for r in ids],
                "positions": list(tx.positions),
                "physical_block_ids": [b for b, _ in tx.locations],
                "block_offsets": [o for _, o in tx.locations],
                "effective_seq_lens": [p + 1 for p in tx.positions],
                "tx_block_tables": [list(r) for r in rows],
            }
            for layer in range(2):
                layer = led.check_layer_for_write(tx, layer)
                led.record_layer_write(tx, layer)
            if step in (4, 11, 20):
                led.abort_token(tx)
                self.snap(f"abort_{step}", extra)
            else:
                led.commit_token(tx)
                self.snap(f"commit_{step}", extra)
            if step == 6:
                led.close_request("b", "finished")
                led.add_request("d")
                self.snap("finish_b_add_d")
            if step == 12:
                led.close_request("a", "cancelled")
                led.add_request("e")
                led.attach_prefix("e", "sys")
                led.add_request("f")
                self.snap("cancel_a_add_e_f")
            if step == 24:
                led.close_request(self.active()[0], "finished")
                self.snap("finish_first")
        try:
            led.evict_prefix("sys")
        except RuntimeError as exc:
            self.log.append({"tag": "evict_refused", "error": str(exc)})
        for rid in self.active():
            led.close_request(rid, "finished")
        self.snap("finish_all")
        released = led.evict_prefix("sys")
        self.snap("evict_prefix", {"released": list(released)})
        small = BlockLedger(num_layers=1, block_size=2, max_blocks=3)
        for rid in (1, 2, 3, 4):
            small.add_request(rid)
        err = None
        try:
            small.begin_token((1, 2, 3, 4))
        except RuntimeError as exc:
            err = str(exc)
        self.log.append({"tag": "capacity_failure", "error": err, "free": list(small.free),
                         "capacity_failure_count": small.metrics(1)["capacity_failure_count"]})
        return self.log


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "ledger_golden.json").read_text())


@pytest.fixture(scope="module")
def replay():
    return _Replay().run()


def test_trace_has_same_steps(golden, replay):
    assert [r["tag"] for r in replay] == [r["tag"] for r in golden]


@pytest.mark.parametrize("idx", range(39))
def test_trace_step_is_bit_exact(idx, golden, replay):
    assert len(golden) == 39
    want, got = golden[idx], replay[idx]
    assert set(got) == set(want), want["tag"]
    for key in want:
        assert got[key] == want[key], f"{want['tag']}: {key}"


def test_ledger_invariants_hold_through_the_trace():
    r = _Replay()
    r.run()
    assert r.ledger.validate_invariants()


def test_request_reactivation_and_duplicate_prefix_ids_are_rejected():
    # reference cache.py:177-190: re-adding an active id is a no-op, a
    # finished/cancelled id cannot come back
    led = BlockLedger(num_layers=1, block_size=4, max_blocks=8, prefix_cache_capacity_blocks=4)
    led.add_request("x")
    version = led.state_version
    led.add_request("x")
    assert led.state_version == version
    led.close_request("x", "finished")
    with pytest.raises(RuntimeError, match="cannot be reactivated"):
        led.add_request("x")
    with pytest.raises(ValueError):
        BlockLedger.check_request_id(["unhashable"])
    block_ids = led.register_prefix("p", 2)
    led.publish_prefix("p", block_ids)
    with pytest.raises(RuntimeError):
        led.register_prefix("p", 1)


def test_abort_returns_boundary_blocks_to_the_front_of_the_free_list():
    led = BlockLedger(num_layers=1, block_size=2, max_blocks=6)
    led.add_request("a")
    led.add_request("b")
    tx = led.begin_token(("a", "b"))
    assert [b for b, _ in tx.locations] == [0, 1]
    led.abort_token(tx)
    assert list(led.free)[:2] == [0, 1]
    assert led.requests["a"].seq_len == 0 and led.requests["a"].block_ids == []


def test_commit_requires_every_layer():
    led = BlockLedger(num_layers=3, block_size=4, max_blocks=4)
    led.add_request("a")
    tx = led.begin_token(("a",))
    led.record_layer_write(tx, led.check_layer_for_write(tx, 0))
    with pytest.raises(RuntimeError):
        led.check_layer_for_write(tx, 2)
    with pytest.raises(RuntimeError):
        led.commit_token(tx)
