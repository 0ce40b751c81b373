"""``flashdec.kernels.paged_decode``: the same module object as
:mod:`flashdec_b200.kernels.paged_decode`."""

import importlib
import sys

sys.modules[__name__] = importlib.import_module("flashdec_b200.kernels.paged_decode")
