"""Host-side behaviour of the Python API that needs no GPU."""
import types

import pytest
import torch

import gemma_triton_flash_attn as gfa
import importlib

att = importlib.import_module("gemma_triton_flash_attn.attention")
from gemma_triton_flash_attn.hf_integration import triton_gqa_attention


def test_public_names_match_reference_api():
    for name in ["attention_flash_gqa", "flash_attn_gqa_train", "FlashAttnGQAFunction", "attention_gqa_ref",
                 "attention_swa_ref", "attention", "register_triton_attention", "triton_gqa_attention",
                 "patch_transformers_5_5_4_flash_attn_key", "patch_gemma4_shared_kv_states_for_fsdp2",
                 "__version__"]:
        assert name in gfa.__all__ and hasattr(gfa, name)


def test_cpu_tensors_fail_loudly_no_fallback():
    q = torch.randn(1, 4, 16, 256, dtype=torch.bfloat16)
    k = torch.randn(1, 2, 16, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        gfa.flash_attn_gqa_train(q, k, k, causal=True)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        gfa.attention_flash_gqa(q, k, k)


@pytest.mark.parametrize("causal,slide,n,expect", [
    (True, 0, 100, 0), (True, 16, 100, 16), (True, 100, 100, 0), (True, 500, 100, 0),
    (False, 16, 100, 0), (True, None, 100, 0),
])
def test_window_normalisation(causal, slide, n, expect):
    assert att._normalize_window(causal, slide, n) == expect


def test_adapter_rejects_softcap_and_dropout():
    mod = types.SimpleNamespace(head_dim=256, is_causal=True)
    q = torch.zeros(1, 2, 8, 256)
    with pytest.raises(NotImplementedError):
        triton_gqa_attention(mod, q, q, q, None, softcap=30.0)
    with pytest.raises(NotImplementedError):
        triton_gqa_attention(mod, q, q, q, None, dropout=0.1)


def test_register_into_transformers_registry():
    pytest.importorskip("transformers")
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    gfa.register_triton_attention("triton_gqa_test")
    assert ALL_ATTENTION_FUNCTIONS["triton_gqa_test"] is triton_gqa_attention


def test_reference_eager_functions_run_on_cpu():
    q = torch.randn(1, 4, 24, 32)
    k = torch.randn(1, 2, 24, 32)
    v = torch.randn(1, 2, 24, 32)
    a = gfa.attention_gqa_ref(q, k, v, causal=True)
    b = gfa.attention_swa_ref(q, k, v, slide_size=24)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


def test_workspace_chunk_plan(monkeypatch):
    """KV heads per chunk of the split materialised backward under a limit
    (workspace linear in B * H_Q; planner allocates on the given device)."""
    from gemma_triton_flash_attn.attention import _workspace_chunks
    size = 2 * 4 * 1000  # B=2, H_KV=4: 1000 bytes per KV head
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", str(size // 3))
    hc, ws = _workspace_chunks(size, 2, 4, "cpu")
    assert hc == 2 and ws.numel() == 2000
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "1500")
    hc, ws = _workspace_chunks(size, 2, 4, "cpu")
    assert hc == 1 and ws.numel() == 1000
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "999")
    assert _workspace_chunks(size, 2, 4, "cpu") == (None, None)
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "0")
    assert _workspace_chunks(size, 2, 4, "cpu") == (None, None)
