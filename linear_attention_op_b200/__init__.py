"""B200-native (sm_100a) Qwen3.5 Gated DeltaNet layer behind a C-ABI (``include/gdn_b200.h``).

The compute lives in ``libgdn_b200.so`` (hand-written CUDA: tcgen05/TMA GEMMs, decode recurrence, conv,
chunked prefill); this package is the host-side mirror of the reference's per-layer op API.
"""

from ._lib import GDNError, GDNLibraryError, device_error, launch_count, lib  # noqa: F401
from .gdn_layer import (  # noqa: F401
    DecoderMlpWeights, GatedDeltaRule, GDNStack, LayerWeights, Qwen35DecoderLayer, Qwen35GatedDeltaNet)

__all__ = ["Qwen35GatedDeltaNet", "Qwen35DecoderLayer", "DecoderMlpWeights", "GDNStack", "GatedDeltaRule",
           "LayerWeights", "GDNError", "GDNLibraryError", "device_error", "launch_count", "lib"]
