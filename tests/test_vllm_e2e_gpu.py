"""vLLM end to end with the flashdec_b200 CUSTOM attention backend.

The backend is loaded the way an installed package provides it: through the
``vllm.general_plugins`` entry point (a temporary dist-info on PYTHONPATH).
A tiny Qwen2-shaped model (16 q heads / 2 KV heads, head_dim 128, dummy
weights) generates greedily from prompts of 520-1200 tokens once with vLLM's
Triton backend and once with CUSTOM; tokens and top logprobs must agree and
the B200 decode kernel must actually have run.

Opt-in (vLLM start-up takes minutes): FD_RUN_VLLM_E2E=1 pytest -m gpu
tests/test_vllm_e2e_gpu.py"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

ROOT = Path(__file__).resolve().parents[1]
CONFIG = {
    "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_size": 2048,
    "intermediate_size": 1024, "num_hidden_layers": 2, "num_attention_heads": 16,
    "num_key_value_heads": 2, "max_position_embeddings": 8192, "rope_theta": 1000000.0,
    "rms_norm_eps": 1e-06, "vocab_size": 1024, "tie_word_embeddings": True,
    "torch_dtype": "bfloat16", "hidden_act": "silu", "use_sliding_window": False,
    "max_window_layers": 2, "bos_token_id": 1, "eos_token_id": 2,
}


@pytest.mark.skipif(os.environ.get("FD_RUN_VLLM_E2E") != "1",
                    reason="opt-in: set FD_RUN_VLLM_E2E=1 (vLLM start-up takes minutes)")
def test_custom_backend_matches_vllm_triton(tmp_path):
    pytest.importorskip("vllm")
    site = tmp_path / "site" / "flashdec_b200-0.1.0.dist-info"
    site.mkdir(parents=True)
    (site / "METADATA").write_text("Metadata-Version: 2.1\nName: flashdec-b200\nVersion: 0.1.0\n")
    (site / "entry_points.txt").write_text(
        "[vllm.general_plugins]\nflashdec_b200 = flashdec_b200.vllm_plugin:register\n")
    model = tmp_path / "model"
    model.mkdir()
    (model / "config.json").write_text(json.dumps(CONFIG))
    env = dict(os.environ, FD_MODEL_DIR=str(model),
               PYTHONPATH=os.pathsep.join([str(tmp_path / "site"), str(ROOT),
                                           os.environ.get("PYTHONPATH", "")]))
    results = {}
    for backend in ("TRITON_ATTN", "CUSTOM"):
        out = tmp_path / f"{backend}.json"
        subprocess.run([sys.executable, "-m", "tests.vllm_e2e_worker", backend, str(out)],
                       cwd=ROOT, env=env, check=True, timeout=900)
        results[backend] = json.loads(out.read_text())
    ref, ours = results["TRITON_ATTN"], results["CUSTOM"]
    assert ours["flashdec_launches"] > 0, "the CUSTOM backend never reached the B200 kernel"
    assert [o["tokens"] for o in ours["outputs"]] == [o["tokens"] for o in ref["outputs"]]
    for a, b in zip(ref["outputs"], ours["outputs"]):
        for la, lb in zip(a["logprobs"], b["logprobs"]):
            for k in set(la) & set(lb):
                assert abs(la[k] - lb[k]) <= 5e-2
