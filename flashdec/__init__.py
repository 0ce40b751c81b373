"""The reference's package name, ``flashdec``, as an alias of
:mod:`flashdec_b200`, so that code written against cysong2025/flashdec runs
unchanged: ``import flashdec``, ``flashdec.decode(...)``,
``flashdec.cache.PagedKVCache``, ``flashdec.engine.DecodeEngine``,
``flashdec.kernels.paged_decode._vllm_paged_decode_attention_into`` and
``flashdec.vllm_backend.FlashDecAttentionBackend`` name the B200
implementation's own objects.

Each submodule of this package is the implementation's module itself (it puts
that module in its place in ``sys.modules``), so classes and functions are
the same objects under both names.  Top-level names resolve on first use, so
importing ``flashdec`` loads no CUDA code.
"""

import flashdec_b200 as _impl

__all__ = list(_impl.__all__)
__version__ = _impl.__version__


def __getattr__(name):
    value = getattr(_impl, name)
    globals()[name] = value
    return value
