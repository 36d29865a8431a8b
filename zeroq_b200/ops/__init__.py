"""Hot ops: each has a PyTorch oracle (CPU) and an sm_100a kernel (CUDA)."""

from .nf4 import (NF4_CODE, FP4_CODE, QuantState, quantize_4bit, dequantize_4bit,
                  quantize_4bit_reference, dequantize_4bit_reference)
from .qlinear import Linear4bit, nf4_linear
from .gemm import gemm_bt
from .norm import add_rmsnorm, rmsnorm
from .rope import apply_rope
from .activations import gelu, swiglu
from .attention import flash_attention
from .cross_entropy import cross_entropy
from .optim import adamw_step, lion_step

__all__ = ["NF4_CODE", "FP4_CODE", "QuantState", "quantize_4bit", "dequantize_4bit",
           "quantize_4bit_reference", "dequantize_4bit_reference", "Linear4bit", "nf4_linear",
           "gemm_bt", "add_rmsnorm", "rmsnorm", "apply_rope", "gelu", "swiglu",
           "flash_attention", "cross_entropy", "adamw_step", "lion_step"]
