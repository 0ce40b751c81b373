"""``flashdec._cuda_kv_append``: the same module object as :mod:`flashdec_b200._cuda_kv_append`."""

import importlib
import sys

sys.modules[__name__] = importlib.import_module("flashdec_b200._cuda_kv_append")
