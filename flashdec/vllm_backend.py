"""``flashdec.vllm_backend``: the same module object as :mod:`flashdec_b200.vllm_backend`."""

import importlib
import sys

sys.modules[__name__] = importlib.import_module("flashdec_b200.vllm_backend")
