from .fused_dequant_attn import (
    fused_dequant_attention,
    fused_dequant_attn_decode,
    fused_dequant_attn_forward,
)
