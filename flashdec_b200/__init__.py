"""flashdec_b200: FlashDec's paged-decode data path, rebuilt for NVIDIA B200.

Public names mirror ``flashdec`` (cysong2025/flashdec ``flashdec/__init__.py``)
for the hot path: ``decode`` / ``paged_decode_attention[_into]``, the fused
RoPE + paged KV append primitives, ``PagedKVCache`` and the
``DecodeEngine`` transaction API.  Imports are lazy so that importing the
package never loads CUDA.  All compute runs in ``libflashdec_b200.so``
(hand-written sm_100a kernels behind a C ABI, ``include/flashdec_b200.h``).
"""

__all__ = [
    "PagedKVCache",
    "KVTokenTransactionView",
    "AdmissionResult",
    "DecodeLayerResult",
    "DecodeEngine",
    "DecodeStepTransaction",
    "DecodeStepResult",
    "RopeAppendResult",
    "__version__",
    "apply_rope",
    "cuda_kv_append",
    "decode",
    "fused_rope_kv_append",
    "load_cuda_kv_append_extension",
    "load_fused_rope_kv_append_extension",
    "paged_decode_attention",
    "paged_decode_attention_into",
    "rope_paged_kv_append",
    "device_status",
    "reserve_workspace",
    "copy_async",
]

__version__ = "0.2.0"

_ENGINE = ("AdmissionResult", "DecodeEngine", "DecodeLayerResult", "DecodeStepResult",
           "DecodeStepTransaction")


def __getattr__(name):
    # resolved once, then a plain module attribute (no import per access:
    # ``flashdec_b200.paged_decode_attention_into`` sits on the per-step path)
    value = _resolve(name)
    globals()[name] = value
    return value


def _resolve(name):
    if name in _ENGINE:
        from . import engine

        return getattr(engine, name)
    if name in ("KVTokenTransactionView", "PagedKVCache"):
        from . import cache

        return getattr(cache, name)
    if name in ("RopeAppendResult", "apply_rope", "rope_paged_kv_append"):
        from . import rope

        return getattr(rope, name)
    if name in ("cuda_kv_append", "load_cuda_kv_append_extension"):
        from . import _cuda_kv_append

        return getattr(_cuda_kv_append, name)
    if name in ("fused_rope_kv_append", "load_fused_rope_kv_append_extension"):
        from . import _fused_rope_kv_append

        return getattr(_fused_rope_kv_append, name)
    if name in ("decode", "paged_decode_attention", "paged_decode_attention_into"):
        from .kernels import paged_decode

        return {
            "decode": paged_decode.paged_decode_attention,
            "paged_decode_attention": paged_decode.paged_decode_attention,
            "paged_decode_attention_into": paged_decode.paged_decode_attention_into,
        }[name]
    if name == "copy_async":
        # the C++ function itself: one cudaMemcpyAsync per call, no Python
        # frame in between (a missing host-path module raises here)
        from ._lib import load_hostpath

        return load_hostpath().copy_async
    if name == "device_status":
        from ._lib import device_status

        return device_status
    if name == "reserve_workspace":
        from ._native import reserve_workspace

        return reserve_workspace
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
