"""``torch.ops.flashdec.*``: the decode calls as PyTorch custom operators.

The public functions (``paged_decode_attention[_into]``, the engine) call the
C ABI directly, which is the cheapest eager path but is opaque to
``torch.compile``: a compiled region that calls them breaks its graph there.
Importing this module registers the same calls as custom operators with fake
(shape-only) implementations, so a model compiled with ``fullgraph=True`` can
contain them:

* ``torch.ops.flashdec.decode(q, k_cache, v_cache, block_tables, seq_lens,
  sm_scale=None, kv_layout="token_major") -> Tensor`` -- reference
  ``flashdec.decode`` (kernels/paged_decode.py:922-969);
* ``torch.ops.flashdec.decode_into(q, k_cache, v_cache, block_tables,
  seq_lens, out, sm_scale=None, kv_layout="token_major") -> ()`` -- reference
  ``paged_decode_attention_into`` (:972-1264), writing ``out``.

Both run the library's launch on the current stream; argument checking and
errors are those of the public functions they call.
"""

from __future__ import annotations

from typing import Optional

import torch

from .kernels import paged_decode as _pd


@torch.library.custom_op("flashdec::decode", mutates_args=())
def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
           block_tables: torch.Tensor, seq_lens: torch.Tensor,
           sm_scale: Optional[float] = None, kv_layout: str = "token_major") -> torch.Tensor:
    return _pd.paged_decode_attention(q, k_cache, v_cache, block_tables, seq_lens,
                                      sm_scale=sm_scale, kv_layout=kv_layout)


@decode.register_fake
def _decode_fake(q, k_cache, v_cache, block_tables, seq_lens, sm_scale=None,
                 kv_layout="token_major"):
    return torch.empty_like(q)


@torch.library.custom_op("flashdec::decode_into", mutates_args=("out",))
def decode_into(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                block_tables: torch.Tensor, seq_lens: torch.Tensor, out: torch.Tensor,
                sm_scale: Optional[float] = None, kv_layout: str = "token_major") -> None:
    _pd.paged_decode_attention_into(q, k_cache, v_cache, block_tables, seq_lens, out,
                                    sm_scale=sm_scale, kv_layout=kv_layout)


@decode_into.register_fake
def _decode_into_fake(q, k_cache, v_cache, block_tables, seq_lens, out, sm_scale=None,
                      kv_layout="token_major"):
    return None
