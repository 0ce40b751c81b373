"""vLLM CUSTOM backend and plugin: identity, split policy (pinned to the
reference's own ``_select_num_splits`` outputs), eligibility and dispatch.

Runs on the CPU: the B200 launcher is replaced by a recorder and vLLM's own
Triton path by a sentinel, so only the host logic is exercised (reference
tests/test_vllm_backend.py, tests/test_vllm_plugin.py)."""

from __future__ import annotations

import json
from types import SimpleNamespace

import pytest
import torch

pytest.importorskip("vllm")

import flashdec_b200.vllm_backend as backend_module  # noqa: E402
from flashdec_b200.vllm_backend import (  # noqa: E402
    FlashDecAttentionBackend,
    FlashDecAttentionImpl,
)
from vllm.v1.attention.backend import AttentionType  # noqa: E402
from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl  # noqa: E402


def test_backend_identity_and_cache_contract():
    assert FlashDecAttentionBackend.get_name() == "CUSTOM"
    assert FlashDecAttentionBackend.get_impl_cls() is FlashDecAttentionImpl
    assert FlashDecAttentionBackend.forward_includes_kv_cache_update is False
    assert FlashDecAttentionBackend.get_kv_cache_shape(7, 16, 2, 128) == (7, 2, 16, 2, 128)


def test_plugin_registers_custom_backend():
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    from flashdec_b200 import vllm_plugin

    try:
        vllm_plugin.register()
        assert AttentionBackendEnum.CUSTOM.get_path() == vllm_plugin.BACKEND_PATH
        assert AttentionBackendEnum.CUSTOM.get_class() is FlashDecAttentionBackend
    finally:
        AttentionBackendEnum.CUSTOM.clear_override()


@pytest.mark.parametrize("value", ["0", "1", "2", "4", "8", "16"])
def test_split_parser_accepts_supported_values(value):
    assert backend_module._parse_requested_splits(value) == int(value)


@pytest.mark.parametrize("value", ["auto", "-1", "3", "6", "11", "12", "17"])
def test_split_parser_rejects_other_values(value):
    with pytest.raises(ValueError, match=r"FLASHDEC_VLLM_NUM_SPLITS must be one of "
                                         r"0, 1, 2, 4, 8, or 16 \(0 selects auto\)"):
        backend_module._parse_requested_splits(value)


def test_split_policy_matches_reference_outputs(golden_dir):
    rows = json.loads((golden_dir / "split_policy_golden.json").read_text())
    assert len(rows) > 4000
    for requested, num_reqs, hkv, logical_blocks, want in rows:
        got = backend_module._select_num_splits(requested, num_reqs=num_reqs, num_kv_heads=hkv,
                                                logical_blocks=logical_blocks)
        assert got == want, (requested, num_reqs, hkv, logical_blocks)


@pytest.mark.parametrize(("num_reqs", "expected"),
                         [(4, 16), (5, 16), (6, 8), (7, 8), (8, 8), (9, 8), (10, 8), (11, 4),
                          (12, 4)])
def test_reference_auto_policy_near_batch_boundaries(num_reqs, expected):
    assert backend_module._select_num_splits(0, num_reqs=num_reqs, num_kv_heads=2,
                                             logical_blocks=64) == expected


def _impl(requested=0, head_size=128):
    impl = object.__new__(FlashDecAttentionImpl)
    impl.num_heads = 16
    impl.num_kv_heads = 2
    impl.head_size = head_size
    impl.scale = head_size ** -0.5
    impl._requested_splits = requested
    impl.attn_type = AttentionType.DECODER
    impl.need_to_return_lse_for_decode = False
    impl.kv_cache_dtype = "auto"
    impl.alibi_slopes = None
    impl.sinks = None
    impl.sliding_window = (-1, -1)
    impl.logits_soft_cap = 0
    return impl


def _metadata(num_reqs=3, max_seq_len=1024, workspace_capacity=64):
    return SimpleNamespace(
        query_start_loc=torch.empty(num_reqs + 1, dtype=torch.int32),
        max_seq_len=max_seq_len, max_query_len=1, use_cascade=False, causal=True,
        block_table=torch.empty((num_reqs, 64), dtype=torch.int32),
        seq_lens=torch.empty(num_reqs, dtype=torch.int32),
        slot_mapping=torch.empty(num_reqs, dtype=torch.int64),
        softmax_segm_output=SimpleNamespace(shape=(workspace_capacity, 16, 16, 128)),
        softmax_segm_max=object(), softmax_segm_expsum=object())


def _tensors(rows=4, dtype=torch.bfloat16, head_size=128, block_size=16):
    q = torch.empty((rows, 16, head_size), dtype=dtype)
    k = torch.empty((rows, 2, head_size), dtype=dtype)
    kv = torch.empty((5, 2, block_size, 2, head_size), dtype=dtype)
    return q, k, torch.empty_like(k), kv, torch.empty_like(q)


@pytest.fixture
def recorder(monkeypatch):
    calls = {"launch": [], "fallback": 0}

    def launch(*args, **kwargs):
        calls["launch"].append((args, kwargs))
        return args[6]

    def fallback(self, *args):
        calls["fallback"] += 1
        return args[6]

    monkeypatch.setattr(backend_module, "_vllm_paged_decode_attention_into", launch)
    monkeypatch.setattr(TritonAttentionImpl, "forward", fallback)
    return calls


def _forward(impl, meta, tensors, **kw):
    q, k, v, kv, out = tensors
    layer = SimpleNamespace(kv_sharing_target_layer_name=None)
    return impl.forward(layer, q, k, v, kv, meta, out, **kw)


def test_auto_mode_runs_the_balanced_b200_schedule_on_original_tensors(recorder):
    impl, meta, t = _impl(0), _metadata(), _tensors()
    assert _forward(impl, meta, t) is t[4]
    assert recorder["fallback"] == 0
    (args, kwargs), = recorder["launch"]
    q, k, v, kv, out = t
    for got, want in zip(args, (q, k, v, kv, meta.block_table, meta.seq_lens, out,
                                meta.slot_mapping, meta.softmax_segm_output,
                                meta.softmax_segm_max, meta.softmax_segm_expsum)):
        assert got is want
    assert kwargs == {"num_reqs": 3, "num_q_heads": 16, "num_kv_heads": 2, "head_dim": 128,
                      "block_size": 16, "sm_scale": 128 ** -0.5, "num_splits": 0}


@pytest.mark.parametrize(("requested", "max_seq_len", "expected"),
                         [(16, 1024, 16), (16, 8192, 16), (8, 512, 8), (16, 100 * 16, 16)])
def test_explicit_splits_follow_the_reference_policy(recorder, requested, max_seq_len,
                                                     expected):
    impl, meta, t = _impl(requested), _metadata(max_seq_len=max_seq_len), _tensors()
    _forward(impl, meta, t)
    assert recorder["launch"][0][1]["num_splits"] == expected


def test_explicit_single_split_and_oversized_batches_use_vllm(recorder):
    _forward(_impl(1), _metadata(), _tensors())
    _forward(_impl(8), _metadata(num_reqs=3, workspace_capacity=2), _tensors())
    assert recorder["launch"] == [] and recorder["fallback"] == 2


@pytest.mark.parametrize("change", [
    dict(meta=dict(max_seq_len=511)), dict(meta=dict(max_query_len=2)),
    dict(meta=dict(use_cascade=True)), dict(meta=dict(causal=False)),
    dict(impl=dict(attn_type=AttentionType.ENCODER)), dict(impl=dict(kv_cache_dtype="fp8")),
    dict(impl=dict(sliding_window=(128, 0))), dict(impl=dict(logits_soft_cap=30.0)),
    dict(impl=dict(alibi_slopes=[1.0])), dict(impl=dict(need_to_return_lse_for_decode=True)),
    dict(impl=dict(num_kv_heads=3)), dict(fp32=True), dict(head_size=96),
    dict(block_size=64), dict(output_scale=True), dict(shared_kv=True),
])
def test_ineligible_calls_go_to_vllm(recorder, change):
    head_size = change.get("head_size", 128)
    impl = _impl(0, head_size=head_size)
    for k, v in change.get("impl", {}).items():
        setattr(impl, k, v)
    meta = _metadata()
    for k, v in change.get("meta", {}).items():
        setattr(meta, k, v)
    t = _tensors(dtype=torch.float32 if change.get("fp32") else torch.bfloat16,
                 head_size=head_size, block_size=change.get("block_size", 16))
    q, k, v, kv, out = t
    layer = SimpleNamespace(kv_sharing_target_layer_name="other" if change.get("shared_kv")
                            else None)
    kw = {"output_scale": torch.ones(1)} if change.get("output_scale") else {}
    impl.forward(layer, q, k, v, kv, meta, out, **kw)
    assert recorder["launch"] == [] and recorder["fallback"] == 1


@pytest.mark.parametrize("head_size,block_size,num_kv_heads", [(64, 8, 2), (128, 32, 1),
                                                               (128, 16, 16)])
def test_wider_shapes_run_on_the_b200_kernel(recorder, head_size, block_size, num_kv_heads):
    impl = _impl(0, head_size=head_size)
    impl.num_kv_heads = num_kv_heads
    q = torch.empty((4, 16, head_size), dtype=torch.float16)
    k = torch.empty((4, num_kv_heads, head_size), dtype=torch.float16)
    kv = torch.empty((5, 2, block_size, num_kv_heads, head_size), dtype=torch.float16)
    impl.forward(SimpleNamespace(kv_sharing_target_layer_name=None), q, k, torch.empty_like(k),
                 kv, _metadata(), torch.empty_like(q))
    assert len(recorder["launch"]) == 1
