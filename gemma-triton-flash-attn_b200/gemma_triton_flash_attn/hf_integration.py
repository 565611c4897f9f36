"""HuggingFace transformers integration (mirror of the reference's
``flash_attn/hf_integration.py``).

    from gemma_triton_flash_attn import register_triton_attention
    register_triton_attention()                      # name "triton_gqa"
    model.config._attn_implementation = "triton_gqa"

Every attention layer of a model that dispatches through transformers'
``ALL_ATTENTION_FUNCTIONS`` then runs the sm_100a kernels.
"""
from __future__ import annotations

import torch

from .attention import FlashAttnGQAFunction, _check_inputs, _fwd, _normalize_window


def _kv_cache_forward(q, k, v, causal, slide, scale):
    _check_inputs(q, k, v, kv_cache=True, causal=causal)
    o, _ = _fwd(q, k, v, causal, _normalize_window(causal, slide, k.shape[2]), scale, want_lse=False)
    return o

__all__ = [
    "triton_gqa_attention",
    "register_triton_attention",
    "patch_transformers_5_5_4_flash_attn_key",
    "patch_gemma4_shared_kv_states_for_fsdp2",
]


def triton_gqa_attention(
    module,
    query: torch.Tensor,            # (B, H_Q, N, D)
    key: torch.Tensor,              # (B, H_KV, N, D)
    value: torch.Tensor,            # (B, H_KV, N, D)
    attention_mask,
    dropout: float = 0.0,
    scaling: float | None = None,
    softcap: float | None = None,
    sliding_window: int | None = None,
    **kwargs,
):
    """transformers ``attention_interface`` adapter (reference: hf_integration.py:30-76).

    Same contract as the reference: ``attention_mask`` is ignored (the kernel
    builds the causal / sliding-window mask from ``module.is_causal`` and
    ``sliding_window``); softcap and non-zero dropout raise NotImplementedError;
    the result is (attn_output of shape (B, N, H_Q, D), None).

    One difference: the reference folds a non-default ``scaling`` into q by a
    separate multiply (hf_integration.py:55-58); here the scale is passed to
    the kernel, which saves a q-sized elementwise pass and the extra rounding
    of q. And because the output keeps the memory layout of ``query`` (HF
    passes a transposed view of (B, N, H, D) storage), the final
    ``transpose(1, 2).contiguous()`` is free.
    """
    if softcap is not None:
        raise NotImplementedError("triton_gqa_attention does not support softcap")
    if dropout != 0.0:
        raise NotImplementedError("triton_gqa_attention does not support dropout")
    scale = scaling if scaling is not None else module.head_dim ** -0.5
    slide = int(sliding_window) if sliding_window else 0
    is_causal = getattr(module, "is_causal", True)
    if key.shape[2] != query.shape[2]:
        # generation with a KV cache: the queries are the last positions of the
        # cache; forward only (the reference reads the wrong key range here,
        # attention.py:552-553)
        if torch.is_grad_enabled() and (query.requires_grad or key.requires_grad or value.requires_grad):
            raise NotImplementedError("triton_gqa_attention: no backward with a KV cache longer than the queries")
        out = _kv_cache_forward(query, key, value, is_causal, slide, float(scale))
    else:
        out = FlashAttnGQAFunction.apply(query, key, value, is_causal, slide, float(scale))
    out = out.transpose(1, 2).contiguous()
    return out, None


def register_triton_attention(name: str = "triton_gqa") -> None:
    """Register the kernel under `name` in transformers' ALL_ATTENTION_FUNCTIONS."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS[name] = triton_gqa_attention


def patch_transformers_5_5_4_flash_attn_key() -> None:
    """Work around transformers 5.5.4's missing "flash_attn" entry in
    PACKAGE_DISTRIBUTION_MAPPING (reference: hf_integration.py:91-99).
    Idempotent; harmless on other versions that have the mapping."""
    try:
        from transformers.utils.import_utils import PACKAGE_DISTRIBUTION_MAPPING
    except ImportError:
        return
    PACKAGE_DISTRIBUTION_MAPPING.setdefault("flash_attn", ["flash-attn"])


def patch_gemma4_shared_kv_states_for_fsdp2() -> None:
    """FSDP2 training glue of the reference (hf_integration.py:102-229).

    Not part of the attention path this library provides; it targets the
    transformers 5.5.4 ``shared_kv_states`` API only.
    """
    raise NotImplementedError(
        "patch_gemma4_shared_kv_states_for_fsdp2 is outside this library's scope "
        "(FSDP2 model glue, not attention)"
    )
