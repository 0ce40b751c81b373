"""The ``flashdec`` package is the reference's import path for this
implementation: every name a reference caller uses resolves to the
flashdec_b200 object itself (not a copy), and importing it loads no CUDA."""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_alias_names_are_the_implementation_objects():
    import flashdec
    import flashdec.cache
    import flashdec.engine
    import flashdec.kernels.paged_decode
    import flashdec.rope
    import flashdec.vllm_plugin
    import flashdec_b200
    import flashdec_b200.cache
    import flashdec_b200.engine
    import flashdec_b200.kernels.paged_decode as pd

    assert flashdec.kernels.paged_decode is pd
    assert flashdec.decode is flashdec_b200.decode
    assert flashdec.paged_decode_attention_into is pd.paged_decode_attention_into
    assert flashdec.kernels.paged_decode._vllm_paged_decode_attention_into is \
        pd._vllm_paged_decode_attention_into
    assert flashdec.cache.PagedKVCache is flashdec_b200.cache.PagedKVCache
    assert flashdec.PagedKVCache is flashdec_b200.PagedKVCache
    assert flashdec.engine.DecodeEngine is flashdec_b200.engine.DecodeEngine
    assert flashdec.rope.apply_rope is flashdec_b200.rope.apply_rope
    assert flashdec.vllm_plugin.register is flashdec_b200.vllm_plugin.register
    assert set(flashdec.__all__) == set(flashdec_b200.__all__)


def test_vllm_backend_path_of_the_reference_resolves():
    pytest.importorskip("vllm")
    import flashdec.vllm_backend
    import flashdec_b200.vllm_backend

    assert flashdec.vllm_backend.FlashDecAttentionBackend is \
        flashdec_b200.vllm_backend.FlashDecAttentionBackend


def test_importing_the_alias_loads_no_torch():
    code = "import sys, flashdec; print('torch' in sys.modules)"
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=120)
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip() == "False"
