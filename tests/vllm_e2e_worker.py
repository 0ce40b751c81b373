"""Worker of tests/test_vllm_e2e_gpu.py: one vLLM generation with a tiny
Qwen2-shaped model (dummy weights) and the given attention backend; writes
tokens, top logprobs and the number of flashdec_b200 launches as JSON.

Run as ``python -m tests.vllm_e2e_worker BACKEND OUT_JSON [eager|graph]``
with FD_MODEL_DIR pointing at the model config directory.  ``graph`` keeps
vLLM's default CUDA-graph mode (decode batches replay FULL graphs, whose
capture goes through the backend's forward); the default is eager."""

from __future__ import annotations

import json
import os
import sys


def main(backend: str, out_path: str, mode: str = "eager") -> None:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # engine core in-process
    import numpy as np
    import torch

    calls = {"n": 0, "captured": 0}
    if backend == "CUSTOM":
        import flashdec_b200.vllm_backend as vb

        orig = vb._vllm_paged_decode_attention_into

        def counted(*a, **k):
            calls["n"] += 1
            if torch.cuda.is_current_stream_capturing():
                calls["captured"] += 1  # this launch is recorded into a CUDA graph
            return orig(*a, **k)

        vb._vllm_paged_decode_attention_into = counted
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    llm = LLM(model=os.environ["FD_MODEL_DIR"], load_format="dummy", skip_tokenizer_init=True,
              dtype="bfloat16", max_model_len=2048, gpu_memory_utilization=0.25,
              attention_backend=backend, seed=0, enforce_eager=(mode != "graph"),
              max_num_seqs=16)
    rng = np.random.default_rng(0)
    lengths = [600, 700, 900, 1200, 520, 800, 1000, 650]  # >= 512: eligible decode batches
    prompts = [TokensPrompt(prompt_token_ids=[int(x) for x in rng.integers(3, 1000, size=n)])
               for n in lengths]
    params = SamplingParams(max_tokens=12, temperature=0.0, logprobs=3, detokenize=False)
    # set only by flashdec_b200.vllm_plugin.register(), which vLLM's own
    # general-plugin loader calls through the installed entry point
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    try:
        custom_path = AttentionBackendEnum.CUSTOM.get_path()
    except ValueError:
        custom_path = ""
    out = []
    for o in llm.generate(prompts, params):
        c = o.outputs[0]
        out.append({"tokens": list(c.token_ids),
                    "logprobs": [{str(k): float(v.logprob) for k, v in d.items()}
                                 for d in (c.logprobs or [])]})
    with open(out_path, "w") as f:
        json.dump({"backend": backend, "mode": mode, "flashdec_launches": calls["n"],
                   "flashdec_captured_launches": calls["captured"], "outputs": out,
                   "plugin_loaded": custom_path.startswith("flashdec_b200.")}, f)


if __name__ == "__main__":
    main(*sys.argv[1:4])
