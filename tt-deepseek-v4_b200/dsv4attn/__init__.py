"""dsv4attn - B200-native (sm_100a) decode sparse-attention path of DeepSeek-V4-Flash.

Layers:
  ``_lib``     ctypes binding of the C ABI (include/dsv4attn.h), no fallback
  ``ops``      torch-tensor wrappers, one per entry point
  ``tables``   rotary / model constants built on the host
  ``layer``    device-resident per-layer state + graph-capturable decode step
  ``modules``  drop-ins keeping the reference's call signatures
  ``dist``     batch split and sequence split across GPUs
"""

from ._lib import NativeLibraryError, lib  # noqa: F401
from .tables import PathArgs  # noqa: F401

__version__ = "0.1.0"
