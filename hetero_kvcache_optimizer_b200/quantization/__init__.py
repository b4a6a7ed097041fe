"""Drop-in for the reference's src/quantization package, whose __init__ exports
KVCompressor (src/quantization/__init__.py:1); PackedKV is this build's packed
INT4 store. The fused attention entry points stay in their modules, as in the
reference: ``quantization.fused_dequant_attn`` (fp32 results) and
``quantization.kernels.fused_dequant_attn`` (q.dtype results)."""
from .kv_compressor import KVCompressor, PackedKV

__all__ = ["KVCompressor", "PackedKV"]
