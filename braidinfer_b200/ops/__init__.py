"""Hot ops.  CUDA tensors run the native sm_100a kernels of ``braidinfer_b200._C``;
CPU tensors run the PyTorch restatements that serve as the test oracle."""
from .attention import AttnMeta, attention, attention_ref, qkv_gemm, qkv_prepare
from .embedding import embedding
from .linear import SWIGLU_BLOCK, gelu_new, interleave_gate_up, linear, linear_swiglu, prefetch_next
from .norm import add_rms_norm, layer_norm, rms_norm, row_rstd
from .rope import apply_rope_ref, build_cos_sin, inv_freq
from .sampling import sample, sample_ref

__all__ = [
    "AttnMeta", "attention", "attention_ref", "qkv_gemm", "qkv_prepare", "embedding", "SWIGLU_BLOCK", "gelu_new",
    "interleave_gate_up", "linear", "linear_swiglu", "prefetch_next", "add_rms_norm", "layer_norm", "rms_norm", "row_rstd",
    "apply_rope_ref", "build_cos_sin", "inv_freq", "sample", "sample_ref",
]
