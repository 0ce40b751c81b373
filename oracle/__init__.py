"""CPU oracle for the FlashDec paged-decode hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``flashdec_b200`` imports this package;
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker
or as the timed CPU baseline -- never as the thing that is measured or shipped.

It is a numpy restatement of the reference's own PyTorch oracles:

* ``paged_attention`` -- ``flashdec/paged_reference.py:19-125``
  (paged single-token decode attention, fp32 math) plus the split-KV
  partial/merge semantics of ``flashdec/kernels/paged_decode.py:330-642``.
* ``rope`` -- ``flashdec/rope.py:26-85`` (split-half RoPE, fp32 math) and the
  slot placement of ``flashdec/csrc/fused_rope_kv_append_kernel.cu:38-82``.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(imported from a checkout of cysong2025/flashdec) on seeded inputs and commits
its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks
this package against every fixture.
"""

from .numerics import bf16_round, fp16_round, round_to_dtype  # noqa: F401
from .paged_attention import (  # noqa: F401
    merge_split_partials,
    paged_decode_attention_ref,
    split_partials_ref,
)
from .rope import apply_rope, inv_freq_table, rope_kv_append_ref  # noqa: F401
