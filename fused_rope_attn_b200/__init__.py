"""B200-native (sm_100a) fused 2D-RoPE + varlen attention forward.

Drop-in for the reference module ``fused_attn`` of sdan/fused-rope-attn
(``fused_rope_attention``, ``compute_rope_2d``) and its ``utils``
(``get_window_index``, ``window_shuffle``, ``window_unshuffle``).
"""
from .fused_attn import (  # noqa: F401
    SUPPORTED_HEAD_DIMS,
    compute_rope_2d,
    fused_attention_rotated,
    fused_rope_attention,
    fused_rope_attention_fp8,
    fused_rope_attention_pos,
    fused_rope_attention_train,
    last_status,
    next_pow2,
    qkv_rope_projection,
    rope_positions_2d,
)

__version__ = "0.1.0"
