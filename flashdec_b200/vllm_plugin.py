"""vLLM general-plugin entry point (reference flashdec/vllm_plugin.py:6-21).

Declare it in the installing package's metadata as
``[project.entry-points."vllm.general_plugins"] flashdec_b200 =
"flashdec_b200.vllm_plugin:register"``; vLLM calls it in the frontend,
engine-core and worker processes.  vLLM is imported only here, so the kernel
and engine API do not depend on it.
"""

from __future__ import annotations

BACKEND_PATH = "flashdec_b200.vllm_backend.FlashDecAttentionBackend"


def register() -> None:
    """Register the B200 backend as vLLM's ``CUSTOM`` attention backend."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.CUSTOM, BACKEND_PATH)
