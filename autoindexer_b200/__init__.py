"""B200-native chain-of-edits (multi-segment RoPE) causal attention.

A drop-in for the fused attention backends of AutodeskAILab/autoindexer
(``autoindexer_triton`` / ``autoindexer_cutedsl``): same transformers
attention-function signature, same position-block input format, computed by
hand-written sm_100a CUDA kernels behind a C ABI (``include/ai_attn.h``).
"""

from .attention import (
    B200_ATTN_KEY,
    AttentionFn,
    attention_interface,
    fused_chain_of_edits_attn_b200,
    read_status,
    register_autoindexer_b200_attention,
    resolve_available_attn_implementation,
)
from .meta import CompiledLayout, RowLayouts, compile_layout
from .positions import (BlockType, PositionBlock, PositionBlockList, blocks_from_concat, cursor_stream,
                        document_blocks, positions_from_operations)
from .decode import decode_attention
from .index_head import compute_index_losses_b200
from .prefill import plain_causal_attn_b200, prefill_attention_interface, prefill_layout
from .rope import SectionedRope, default_inv_freq

__all__ = [
    "B200_ATTN_KEY",
    "AttentionFn",
    "attention_interface",
    "fused_chain_of_edits_attn_b200",
    "read_status",
    "register_autoindexer_b200_attention",
    "resolve_available_attn_implementation",
    "CompiledLayout",
    "RowLayouts",
    "compile_layout",
    "BlockType",
    "PositionBlock",
    "PositionBlockList",
    "cursor_stream",
    "document_blocks",
    "blocks_from_concat",
    "positions_from_operations",
    "decode_attention",
    "compute_index_losses_b200",
    "plain_causal_attn_b200",
    "prefill_attention_interface",
    "prefill_layout",
    "SectionedRope",
    "default_inv_freq",
]
