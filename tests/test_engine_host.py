"""DecodeEngine / PagedKVCache host logic on the CPU (no kernel runs).

A CPU-resident cache keeps every integer decision but refuses data writes
(there is no CPU data path), which lets these tests drive the lifecycle, the
transaction bookkeeping and the abort-on-failure contract of reference
engine.py:594-752 without a GPU."""

from __future__ import annotations

import pytest
import torch

from flashdec_b200.cache import PagedKVCache
from flashdec_b200.engine import (
    AdmissionResult,
    DecodeEngine,
    DecodeStepResult,
    DecodeStepTransaction,
)


def _cache(num_layers=2, max_blocks=16, block_size=4):
    return PagedKVCache(num_layers=num_layers, num_kv_heads=2, head_dim=8, block_size=block_size,
                        max_blocks=max_blocks, dtype=torch.bfloat16, device="cpu")


def _qkv(n, hq=4):
    return (torch.zeros((n, hq, 8), dtype=torch.bfloat16),
            torch.zeros((n, 2, 8), dtype=torch.bfloat16),
            torch.zeros((n, 2, 8), dtype=torch.bfloat16))


def test_constructor_validation():
    with pytest.raises(TypeError, match="PagedKVCache"):
        DecodeEngine(object())
    with pytest.raises(ValueError, match="append_backend"):
        DecodeEngine(_cache(), append_backend="triton")
    with pytest.raises(ValueError, match="CPU semantic oracle"):
        DecodeEngine(_cache(), decode_backend="reference")
    with pytest.raises(ValueError, match="decode_backend"):
        DecodeEngine(_cache(), decode_backend="flashinfer")
    with pytest.raises(ValueError, match="profile_ranges"):
        DecodeEngine(_cache(), profile_ranges=1)
    assert DecodeEngine(_cache(), decode_backend="triton").decode_backend == "triton"


def test_request_lifecycle_and_metrics():
    eng = DecodeEngine(_cache())
    assert eng.add_request("a") == AdmissionResult("a", "waiting")
    eng.add_request("b")
    with pytest.raises(RuntimeError, match="already exists"):
        eng.add_request("a")
    with pytest.raises(ValueError, match="hashable"):
        eng.add_request(["x"])
    assert eng.request_state("a") == {"request_id": "a", "status": "waiting"}
    assert eng.admit(["b"]) == (AdmissionResult("b", "active"),)
    assert eng.admit() == (AdmissionResult("a", "active"),)
    with pytest.raises(ValueError, match="at least one waiting"):
        eng.admit()
    # submission order, as the reference's status dict iterates
    assert eng.active_request_ids() == ("a", "b")
    assert eng.request_state("a")["cache"]["seq_len"] == 0
    eng.finish_request("b")
    eng.add_request("c")
    eng.admit("c")
    eng.cancel_request("c")
    with pytest.raises(RuntimeError, match="is finished, expected active"):
        eng.finish_request("b")
    with pytest.raises(KeyError):
        eng.request_state("zzz")
    m = eng.metrics()
    assert (m["waiting_requests"], m["active_requests"], m["finished_requests"],
            m["cancelled_requests"]) == (0, 1, 1, 1)
    assert m["scheduler_managed"] is False and m["decode_backend"] == "cuda"
    assert m["cache"]["active_requests"] == 1
    assert eng.validate_invariants()


def test_scheduler_mode_is_out_of_scope():
    eng = DecodeEngine(_cache())
    for call in (lambda: eng.submit_request(object()), lambda: eng.scheduling_snapshot(0),
                 lambda: eng.prefill_request("a", None, None),
                 lambda: eng.prefill_request_layers("a", None, None),
                 lambda: eng.apply_scheduler_decision(None, scheduler=None, snapshot=None)):
        with pytest.raises(NotImplementedError, match="scheduler-managed"):
            call()


def test_begin_step_reserves_slots_and_a_failing_layer_aborts_the_token():
    cache = _cache()
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    for rid in ("a", "b"):
        eng.add_request(rid)
    eng.admit()
    free_before = cache.num_free_blocks
    tx = eng.begin_step()
    assert isinstance(tx, DecodeStepTransaction)
    assert tx.request_ids == ("a", "b")
    assert tx.positions.tolist() == [0, 0]
    assert tx.physical_block_ids.tolist() == [0, 1]
    assert tx.block_offsets.tolist() == [0, 0]
    assert tx.effective_seq_lens.tolist() == [1, 1]
    assert cache.num_free_blocks == free_before - 2
    with pytest.raises(RuntimeError, match="during an open decode step"):
        eng.add_request("c")
    with pytest.raises(RuntimeError, match="before all layers"):
        eng.commit_step(tx)
    assert eng.validate_invariants()
    # the CPU cache refuses the data write -> the whole token is aborted
    with pytest.raises(ValueError, match="CUDA-resident"):
        eng.step_layer(tx, 0, *_qkv(2))
    assert not cache.has_open_transaction
    assert cache.num_free_blocks == free_before
    assert eng.metrics()["transaction_abort_count"] == 1
    assert eng.request_state("a")["cache"]["seq_len"] == 0
    with pytest.raises(RuntimeError, match="no open decode step"):
        eng.abort_step(tx)
    # the same slots are reserved again by the next token
    tx2 = eng.begin_step()
    assert tx2.physical_block_ids.tolist() == [0, 1]
    assert eng.abort_step(tx2).state == "aborted"
    assert eng.validate_invariants()


def test_layer_order_shape_checks_and_stale_handles_abort():
    eng = DecodeEngine(_cache(), append_backend="torch")
    eng.add_request("a")
    eng.admit()
    tx = eng.begin_step()
    with pytest.raises(RuntimeError, match="requires layer 0, got layer 1"):
        eng.step_layer(tx, 1, *_qkv(1))
    assert eng.metrics()["transaction_abort_count"] == 1
    tx = eng.begin_step()
    q, k, v = _qkv(1)
    with pytest.raises(ValueError, match="q shape"):
        eng.step_layer(tx, 0, q[:, :, :4], k, v)
    tx = eng.begin_step()
    with pytest.raises(ValueError, match="dtype"):
        eng.step_layer(tx, 0, q.float(), k, v)
    tx = eng.begin_step()
    forged = DecodeStepTransaction(tx.transaction_id, tx.engine_version + 1, tx.request_ids,
                                   None, None, None, None, None)
    with pytest.raises(RuntimeError, match="stale or invalid"):
        eng.step_layer(forged, 0, q, k, v)
    with pytest.raises(TypeError):
        eng.commit_step("not a handle")
    eng.abort_step(tx)
    assert eng.validate_invariants()


def test_multi_layer_transactions_need_a_transaction_backend():
    eng = DecodeEngine(_cache(), append_backend="cuda")
    eng.add_request("a")
    eng.admit()
    with pytest.raises(RuntimeError, match="multi-layer transactions require"):
        eng.begin_step()


def test_single_layer_step_reports_backpressure_without_state_change():
    cache = _cache(num_layers=1, max_blocks=1)
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    for rid in ("a", "b"):
        eng.add_request(rid)
    eng.admit()
    version = cache.state_version
    res = eng.step(*_qkv(2))
    assert isinstance(res, DecodeStepResult)
    assert res.status == "backpressure" and res.reason == "insufficient_physical_blocks"
    assert res.needed_new_blocks == 2 and res.free_blocks == 1 and res.output is None
    assert cache.state_version == version
    assert eng.metrics()["backpressure_count"] == 1
    with pytest.raises(RuntimeError, match="insufficient physical blocks"):
        eng.begin_step()
    with pytest.raises(RuntimeError, match="multi-layer caches"):
        DecodeEngine(_cache(num_layers=2)).step(*_qkv(1))


def test_prefix_registration_rules():
    cache = PagedKVCache(num_layers=2, num_kv_heads=2, head_dim=8, block_size=4, max_blocks=8,
                         dtype=torch.bfloat16, device="cpu", prefix_cache_capacity_blocks=2)
    eng = DecodeEngine(cache)
    blocks = torch.zeros((2, 1, 2, 4, 8), dtype=torch.bfloat16)
    # index_copy_ of the prefix blocks is a plain tensor copy and works on CPU
    state = eng.register_prefix("sys", blocks, blocks)
    assert state["num_blocks"] == 1
    eng.add_request("a")
    with pytest.raises(RuntimeError, match="before request submission"):
        eng.register_prefix("p2", blocks, blocks)
    eng.admit()
    with pytest.raises(RuntimeError, match="after all requests are resolved"):
        eng.evict_prefix("sys")
    eng.finish_request("a")
    assert list(eng.evict_prefix("sys")) == [0]
