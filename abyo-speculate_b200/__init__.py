"""B200-native backend for abyo-speculate's target-model verify step.

Import with ``importlib.import_module("abyo-speculate_b200")`` (the directory
name carries a hyphen).  The compute path is ``libspecb200.so`` (sm_100a CUDA
kernels behind the C ABI in include/spec_b200.h); this package is the host
mirror of the reference's Decoder / TreeDecoder interface.
"""

from ._lib import (CacheRollbackError, DeviceError, IoError, SamplingError, SpecError,  # noqa: F401
                   UnsupportedMethodError, LIB_PATH, MAX_ROWS, load)
from .decoder import B200Decoder, QWeight, exchange_tp_handles  # noqa: F401
from .tree import DraftTree  # noqa: F401

__all__ = [
    "B200Decoder", "QWeight", "DraftTree", "SpecError", "SamplingError", "CacheRollbackError",
    "UnsupportedMethodError", "IoError", "DeviceError", "LIB_PATH", "MAX_ROWS", "load", "exchange_tp_handles",
]
