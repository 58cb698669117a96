"""Blockwise FP8 kernels on sm_100a, with the export list of the reference's
ltx-kernels/src/ltx_kernels/blockwise/__init__.py."""
from ltx_kernels.blockwise.functional import (
    blockwise_dequantize,
    blockwise_quantize_adanorm_triton,
    blockwise_quantize_rms_fma_triton,
    fp6_blockwise_quantize_weights_torch,
    fp6_pack_tensor,
    fp6_unpack_tensor,
    fp8_blockwise_quantize_weights_torch,
    gated_attention_triton,
    rms_norm_rope,
    rms_norm_split_rope,
)
from ltx_kernels.blockwise.linear import BlockwiseFP6Linear, BlockwiseFP8Linear
from ltx_kernels.blockwise.fused import BlockwiseFP8FeedForward, BlockwiseFP8LoRALinear, fp8_linear
from ltx_kernels.blockwise.lora_fuse import blockwise_fp8_fuse, blockwise_fp8_fuse_rule, merge_loras
from ltx_kernels.blockwise.host_stream import TokenStreamer, stream_tokens

__all__ = [
    "BlockwiseFP6Linear",
    "BlockwiseFP8Linear",
    "BlockwiseFP8FeedForward",
    "BlockwiseFP8LoRALinear",
    "TokenStreamer",
    "blockwise_dequantize",
    "blockwise_fp8_fuse",
    "blockwise_fp8_fuse_rule",
    "merge_loras",
    "blockwise_quantize_adanorm_triton",
    "blockwise_quantize_rms_fma_triton",
    "fp6_blockwise_quantize_weights_torch",
    "fp6_pack_tensor",
    "fp6_unpack_tensor",
    "fp8_blockwise_quantize_weights_torch",
    "fp8_linear",
    "gated_attention_triton",
    "rms_norm_rope",
    "rms_norm_split_rope",
    "stream_tokens",
]
