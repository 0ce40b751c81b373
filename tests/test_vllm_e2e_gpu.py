"""vLLM end to end with the flashdec_b200 CUSTOM attention backend.

The backend is loaded the way an installed package provides it: pip builds
the repository's own ``pyproject.toml`` into a temporary target directory,
and vLLM finds ``flashdec_b200.vllm_plugin:register`` through the
``vllm.general_plugins`` entry point of that install's metadata.  The
in-tree package stays first on ``PYTHONPATH`` so the in-tree sm_100a library
is the one loaded.  A tiny Qwen2-shaped model (16 q heads / 2 KV heads,
head_dim 128, dummy weights) generates greedily from prompts of 520-1200
tokens once with vLLM's Triton backend and once with CUSTOM; tokens and top
logprobs must agree and the B200 decode kernel must actually have run.  The
pair runs twice: eager, and in vLLM's default CUDA-graph mode, where the
decode batches replay FULL graphs whose capture recorded the B200 kernel.

Runs by default under ``-m gpu`` (four vLLM start-ups, a few minutes);
FD_SKIP_VLLM_E2E=1 skips it."""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
import time
from pathlib import Path

import pytest

pytestmark = [pytest.mark.gpu]

ROOT = Path(__file__).resolve().parents[1]
CONFIG = {
    "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_size": 2048,
    "intermediate_size": 1024, "num_hidden_layers": 2, "num_attention_heads": 16,
    "num_key_value_heads": 2, "max_position_embeddings": 8192, "rope_theta": 1000000.0,
    "rms_norm_eps": 1e-06, "vocab_size": 1024, "tie_word_embeddings": True,
    "torch_dtype": "bfloat16", "hidden_act": "silu", "use_sliding_window": False,
    "max_window_layers": 2, "bos_token_id": 1, "eos_token_id": 2,
}


def _install_package(tmp_path: Path) -> Path:
    """pip-install the repository (pyproject.toml) into a target directory,
    from a copy so the build writes nothing into the source tree."""
    src = tmp_path / "src"
    src.mkdir()
    shutil.copy(ROOT / "pyproject.toml", src / "pyproject.toml")
    shutil.copytree(ROOT / "flashdec_b200", src / "flashdec_b200",
                    ignore=shutil.ignore_patterns("__pycache__", "_build", "csrc"))
    shutil.copytree(ROOT / "flashdec", src / "flashdec",
                    ignore=shutil.ignore_patterns("__pycache__"))
    site = tmp_path / "site"
    subprocess.run([sys.executable, "-m", "pip", "install", "--quiet", "--no-index",
                    "--no-deps", "--no-build-isolation", "--target", str(site), str(src)],
                   check=True, timeout=600)
    eps = list(site.glob("flashdec_b200-*.dist-info/entry_points.txt"))
    assert eps, "pip produced no entry_points.txt for flashdec_b200"
    text = eps[0].read_text()
    assert "[vllm.general_plugins]" in text and "flashdec_b200.vllm_plugin:register" in text
    return site


@pytest.fixture(scope="module")
def installed(tmp_path_factory):
    if os.environ.get("FD_SKIP_VLLM_E2E") == "1":
        pytest.skip("FD_SKIP_VLLM_E2E=1")
    pytest.importorskip("vllm")
    tmp = tmp_path_factory.mktemp("vllm_e2e")
    site = _install_package(tmp)
    model = tmp / "model"
    model.mkdir()
    (model / "config.json").write_text(json.dumps(CONFIG))
    return tmp, site, model


@pytest.mark.parametrize("mode", ["eager", "graph"])
def test_custom_backend_matches_vllm_triton(installed, mode):
    tmp, site, model = installed
    env = dict(os.environ, FD_MODEL_DIR=str(model),
               PYTHONPATH=os.pathsep.join([str(ROOT), str(site),
                                           os.environ.get("PYTHONPATH", "")]))
    results, seconds = {}, {}
    for backend in ("TRITON_ATTN", "CUSTOM"):
        out = tmp / f"{backend}_{mode}.json"
        t0 = time.monotonic()
        subprocess.run([sys.executable, "-m", "tests.vllm_e2e_worker", backend, str(out), mode],
                       cwd=ROOT, env=env, check=True, timeout=900)
        seconds[backend] = time.monotonic() - t0
        results[backend] = json.loads(out.read_text())
    print(f"vLLM e2e ({mode}) wall seconds: {seconds}")
    ref, ours = results["TRITON_ATTN"], results["CUSTOM"]
    assert ours["plugin_loaded"], "vLLM did not load flashdec_b200 through its entry point"
    assert ours["flashdec_launches"] > 0, "the CUSTOM backend never reached the B200 kernel"
    if mode == "graph":
        assert ours["flashdec_captured_launches"] > 0, "no FULL graph recorded the B200 kernel"
    assert [o["tokens"] for o in ours["outputs"]] == [o["tokens"] for o in ref["outputs"]]
    for a, b in zip(ref["outputs"], ours["outputs"]):
        for la, lb in zip(a["logprobs"], b["logprobs"]):
            for k in set(la) & set(lb):
                assert abs(la[k] - lb[k]) <= 5e-2
