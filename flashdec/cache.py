"""``flashdec.cache``: the same module object as :mod:`flashdec_b200.cache`."""

import importlib
import sys

sys.modules[__name__] = importlib.import_module("flashdec_b200.cache")
