"""usaf_b200: B200-native (sm_100a) MoE expert hot path of USAF.

Drop-in counterparts of the reference's hot-path API:
  usaf_b200.quantization   quantize_4bit / dequantize_4bit (packed int4, device)
  usaf_b200.moe_loader     QuantizedExpertCache, SparseGradStore, TopKImportanceStore
  usaf_b200.sparse_optim   SparseAdam (device state, fused kernel)
  usaf_b200.selector       TopKSelector, ThresholdSelector, DynamicSelector
  usaf_b200.qwen3moe       patch_qwen3moe_for_b200 (Qwen3-MoE block forward/backward)
Engine: usaf_b200.engine (Projection, MoEBlock) over the C ABI in
include/usaf_b200.h, loaded from the in-tree libusaf_b200.so.
"""
from . import _lib  # noqa: F401  (fails loudly when the native library is missing)

__version__ = "0.1.0"
