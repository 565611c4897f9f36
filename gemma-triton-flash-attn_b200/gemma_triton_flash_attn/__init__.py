"""gemma_triton_flash_attn (B200 edition): GQA flash attention for Gemma-4
shapes (head_dim 512 full causal, head_dim 256 sliding window) on sm_100a.

Drop-in for the reference package of the same import name: same public names
and semantics, hand-written tcgen05/TMA kernels behind a C ABI instead of
Triton. See ``attention`` and ``hf_integration`` for the API.
"""
from .attention import (
    attention_flash_gqa,
    flash_attn_gqa_train,
    FlashAttnGQAFunction,
    attention_gqa_ref,
    attention_swa_ref,
    attention,
    flash_attn_gqa_forward_with_lse,
    flash_attn_gqa_backward,
)
from .hf_integration import (
    register_triton_attention,
    triton_gqa_attention,
    patch_transformers_5_5_4_flash_attn_key,
    patch_gemma4_shared_kv_states_for_fsdp2,
)

__version__ = "0.1.0"

__all__ = [
    "attention_flash_gqa",
    "flash_attn_gqa_train",
    "FlashAttnGQAFunction",
    "attention_gqa_ref",
    "attention_swa_ref",
    "attention",
    "register_triton_attention",
    "triton_gqa_attention",
    "patch_transformers_5_5_4_flash_attn_key",
    "patch_gemma4_shared_kv_states_for_fsdp2",
    "__version__",
]
