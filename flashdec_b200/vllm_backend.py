"""Out-of-tree vLLM attention backend backed by the B200 decode kernels.

Drop-in for ``flashdec/vllm_backend.py`` (cysong2025/flashdec): the same
classes, registration name (``CUSTOM``), KV-cache contract
(``forward_includes_kv_cache_update = False``: vLLM keeps its own KV update
op, the fused kernel stores the current token again) and the same
``FLASHDEC_VLLM_NUM_SPLITS`` switch.  vLLM keeps ownership of cache
allocation, metadata, prefill, mixed batches and every feature outside
uniform single-token decoder attention over an fp16/bf16 paged cache; those
batches go to vLLM's Triton implementation (the parent class).

Split policy:

* ``FLASHDEC_VLLM_NUM_SPLITS=0`` (default, auto): one launch of the
  length-balanced B200 schedule, partials merged inside the kernel
  (``num_splits=0`` of the launcher).  The schedule reads the true lengths on
  the device, so no host value is needed and the call is CUDA-graph safe
  once the per-device workspace has been sized by an eager call (vLLM's
  warm-up runs do that) or by ``flashdec_b200.reserve_workspace``.
* ``1``: vLLM's own Triton path, as in the reference.
* ``2, 4, 8, 16``: the reference policy (:func:`_select_num_splits`,
  vllm_backend.py:168-188: capped at the largest legal split not above the
  logical block count) with vLLM's ``softmax_segm_*`` buffers as the split
  workspace, followed by the split reducer; batches larger than those
  buffers fall back to one split (vLLM's path), as the reference does.
"""

from __future__ import annotations

import os

import torch

from vllm.v1.attention.backend import AttentionType
from vllm.v1.attention.backends.triton_attn import (
    TritonAttentionBackend,
    TritonAttentionImpl,
    TritonAttentionMetadata,
)

from .kernels.paged_decode import _vllm_paged_decode_attention_into

_VALID_REQUESTED_SPLITS = (0, 1, 2, 4, 8, 16)
_VALID_NUM_SPLITS = _VALID_REQUESTED_SPLITS[1:]


def _parse_requested_splits(value: str) -> int:
    """``FLASHDEC_VLLM_NUM_SPLITS`` value -> requested split count (0 = auto)."""
    try:
        requested = int(value)
    except ValueError:
        requested = -1
    if requested not in _VALID_REQUESTED_SPLITS:
        raise ValueError("FLASHDEC_VLLM_NUM_SPLITS must be one of 0, 1, 2, 4, 8, or 16 "
                         "(0 selects auto)")
    return requested


def _select_num_splits(requested_splits: int, *, num_reqs: int, num_kv_heads: int,
                       logical_blocks: int) -> int:
    """The reference's split policy (vllm_backend.py:168-188).

    The cap is the largest legal split count not above the logical block
    count; ``requested_splits == 0`` picks the legal count whose program
    count ``num_reqs * num_kv_heads * split`` is nearest to 128 (ties to the
    smaller split)."""
    cap = max(s for s in _VALID_NUM_SPLITS if s <= max(1, logical_blocks))
    if requested_splits == 0:
        per_split = max(1, num_reqs * num_kv_heads)
        requested_splits = min(_VALID_NUM_SPLITS, key=lambda s: (abs(per_split * s - 128), s))
    return min(requested_splits, cap)


class FlashDecAttentionBackend(TritonAttentionBackend):
    """vLLM backend that runs eligible decode batches on the B200 kernels."""

    forward_includes_kv_cache_update = False

    @staticmethod
    def get_name() -> str:
        # vLLM maps the selected class back through its registry by name, so
        # a third-party backend reports the enum slot it is registered in.
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["FlashDecAttentionImpl"]:
        return FlashDecAttentionImpl


class FlashDecAttentionImpl(TritonAttentionImpl):
    """B200 kernels for the decode path they implement; vLLM for the rest."""

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        self._requested_splits = _parse_requested_splits(
            os.environ.get("FLASHDEC_VLLM_NUM_SPLITS", "0"))

    def _supports_flashdec_decode(self, query, key, value, kv_cache, attn_metadata, output,
                                  output_scale, output_block_scale) -> bool:
        """Eligibility of one forward call (reference vllm_backend.py:225-289,
        widened to every head size / page size / GQA group the kernel runs)."""
        if attn_metadata is None:
            return False
        if self.attn_type != AttentionType.DECODER:
            return False
        if attn_metadata.max_seq_len < 512:
            return False
        if attn_metadata.max_query_len != 1 or attn_metadata.use_cascade:
            return False
        if getattr(attn_metadata, "causal", True) is not True:
            return False
        if self.need_to_return_lse_for_decode:
            return False
        if output_scale is not None or output_block_scale is not None:
            return False
        if self.kv_cache_dtype not in ("auto", "float16", "bfloat16"):
            return False
        if query.dtype not in (torch.float16, torch.bfloat16) or kv_cache.dtype != query.dtype:
            return False
        if query.ndim != 3 or key.ndim != 3 or value.ndim != 3 or output.ndim != 3:
            return False
        if kv_cache.ndim != 5:
            return False
        if self.head_size not in (64, 128):
            return False
        if (kv_cache.shape[1] != 2 or kv_cache.shape[2] not in (8, 16, 32)
                or kv_cache.shape[3] != self.num_kv_heads or kv_cache.shape[4] != self.head_size):
            return False
        if self.alibi_slopes is not None or self.sinks is not None:
            return False
        if self.sliding_window != (-1, -1) or self.logits_soft_cap != 0:
            return False
        return self.num_heads % self.num_kv_heads == 0

    def forward(self, layer, query, key, value, kv_cache, attn_metadata: TritonAttentionMetadata,
                output, output_scale=None, output_block_scale=None):
        owns_kv = (getattr(layer, "kv_sharing_target_layer_name", None) is None
                   and key is not None and value is not None)
        if not owns_kv or not self._supports_flashdec_decode(
                query, key, value, kv_cache, attn_metadata, output, output_scale,
                output_block_scale):
            return super().forward(layer, query, key, value, kv_cache, attn_metadata, output,
                                   output_scale, output_block_scale)

        # One query token per metadata row; under CUDA-graph replay the row
        # count includes padding rows, whose slot_mapping is -1 (zero output,
        # no store) so no device value is read on the host.
        num_reqs = attn_metadata.query_start_loc.shape[0] - 1
        block_size = kv_cache.shape[2]
        if self._requested_splits == 0:
            num_splits = 0
        else:
            logical_blocks = (attn_metadata.max_seq_len + block_size - 1) // block_size
            num_splits = _select_num_splits(self._requested_splits, num_reqs=num_reqs,
                                            num_kv_heads=self.num_kv_heads,
                                            logical_blocks=logical_blocks)
            if num_reqs > attn_metadata.softmax_segm_output.shape[0]:
                num_splits = 1
            if num_splits == 1:
                return super().forward(layer, query, key, value, kv_cache, attn_metadata,
                                       output, output_scale, output_block_scale)
        _vllm_paged_decode_attention_into(
            query, key, value, kv_cache, attn_metadata.block_table, attn_metadata.seq_lens,
            output, attn_metadata.slot_mapping, attn_metadata.softmax_segm_output,
            attn_metadata.softmax_segm_max, attn_metadata.softmax_segm_expsum,
            num_reqs=num_reqs, num_q_heads=self.num_heads, num_kv_heads=self.num_kv_heads,
            head_dim=self.head_size, block_size=block_size, sm_scale=self.scale,
            num_splits=num_splits)
        return output
