"""Pinned native 48 kHz stereo checkpoint and its mixed-precision policy.

Same checkpoint, revision, precision policy and weight layout as
fast_moss/v2_loading.py:7-45 (FP32 parameters, BF16 compute, FP32
quantizer, SDPA attention); the B200 path changes no weight.
"""

import torch

MODEL_ID = "OpenMOSS-Team/MOSS-Audio-Tokenizer-v2"
REVISION = "f6e20e543b33d2c252a7ef71bdf8aa71e5ff9169"


def strict_precision():
    """Keep the native FP32 operations free of TF32 approximation."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")


def load_model(device="cuda", *, attention_implementation="sdpa", compute_dtype="bf16"):
    """Loads the pinned checkpoint with FP32 parameters (reference
    fast_moss/v2_loading.py:18-45)."""
    if attention_implementation not in ("sdpa", "flash_attention_2"):
        raise ValueError("Unknown v2 attention implementation")
    if compute_dtype not in ("bf16", "fp32"):
        raise ValueError("Unknown v2 compute dtype")
    strict_precision()
    from transformers import AutoModel

    with torch.inference_mode(False):
        return (
            AutoModel.from_pretrained(
                MODEL_ID,
                revision=REVISION,
                trust_remote_code=True,
                dtype=torch.float32,
                codec_weight_dtype="fp32",
                attention_implementation=attention_implementation,
                compute_dtype=compute_dtype,
            )
            .eval()
            .to(device)
            .requires_grad_(False)
        )
