"""Kernel-level entry points (``flashdec.kernels`` counterpart for the hot path)."""

__all__ = ["paged_decode_attention", "paged_decode_attention_into"]


def paged_decode_attention(*args, **kwargs):
    """Lazily dispatch to the B200 paged decode attention."""
    from .paged_decode import paged_decode_attention as _impl

    return _impl(*args, **kwargs)


def paged_decode_attention_into(*args, **kwargs):
    from .paged_decode import paged_decode_attention_into as _impl

    return _impl(*args, **kwargs)
