"""B200-native hot path of the MOSS Audio Tokenizer v2 codec.

Drop-in for the data-parallel hot path of fast_moss (kadirnar/fast-moss-tokenizer):
the same kernel-level functions (`rotate`, `scale_add`, `select`, `prepare`)
and entry points (`optimized`, `StreamingCodec`, `codec`, `encode_fixed`,
`load_model`) backed by hand-written sm_100a CUDA kernels in
libfast_moss_b200.so, plus
the fused forms (residual + LayerNorm, in-kernel RoPE phase, gated
activation, fused LFQ decode, the whole multi-stage residual VQ in one
kernel, the real codec's 32-stage LFQ loop in one kernel, a tcgen05 Linear
with its activation epilogue), and the streaming transformer stack with
its batched CUDA-graph scheduler (`StreamingTransformer`, `BatchedStreams`).
"""

from . import _lib
from .graphs import CapturedStep, GraphedCallable
from .lfq_rvq import LFQResidualQuantizer
from .linear import PackedWeight, linear, pack_weight
from .quantizer import decode_latents, select
from .quantizer_prepare import prepare
from .rvq import ResidualVectorQuantizer
from .v2_pointwise import (
    gated_activation,
    history_attention,
    history_attention_qkv,
    layer_norm,
    pack_qkv_weight,
    qkv_rope,
    residual_layer_norm,
    rope,
    rope_kv,
    rotate,
    scale_add,
)
from .streaming import StreamingCodec
from .transformer import BatchedStreams, StackConfig, StreamingTransformer
from .v2_codec import codec, encode_fixed
from .v2_loading import load_model
from .v2_runtime import V2Runtime, optimized, validate

__all__ = [
    "rotate",
    "rope",
    "rope_kv",
    "pack_qkv_weight",
    "qkv_rope",
    "scale_add",
    "layer_norm",
    "residual_layer_norm",
    "gated_activation",
    "history_attention",
    "history_attention_qkv",
    "select",
    "decode_latents",
    "prepare",
    "ResidualVectorQuantizer",
    "GraphedCallable",
    "CapturedStep",
    "LFQResidualQuantizer",
    "linear",
    "pack_weight",
    "PackedWeight",
    "StreamingCodec",
    "StackConfig",
    "StreamingTransformer",
    "BatchedStreams",
    "codec",
    "encode_fixed",
    "load_model",
    "optimized",
    "V2Runtime",
    "validate",
]


def library_path():
    """Path of the native library that every op of this package calls."""
    return _lib.LIB_PATH
