"""``flashdec.kernels``: the kernel API of :mod:`flashdec_b200.kernels`."""

import flashdec_b200.kernels as _impl

__all__ = list(_impl.__all__)


def __getattr__(name):
    return getattr(_impl, name)
