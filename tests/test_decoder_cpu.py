"""The synthetic Gemma-4-shaped decoder (config 5) dispatches attention through
transformers' registry with HF's calling convention. CPU check of the plumbing
with an explicit-math attention function standing in for the kernel."""
import pytest
import torch

pytest.importorskip("transformers")
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS  # noqa: E402

from gemma_triton_flash_attn.gemma4_synthetic import Gemma4SyntheticConfig, Gemma4SyntheticDecoder  # noqa: E402

CALLS = []


def explicit_attention(module, q, k, v, mask, dropout=0.0, scaling=None, sliding_window=None, **kw):
    CALLS.append((q.shape, k.shape, scaling, sliding_window, q.is_contiguous()))
    g = q.shape[1] // k.shape[1]
    kk, vv = k.repeat_interleave(g, 1).float(), v.repeat_interleave(g, 1).float()
    s = (q.float() @ kk.transpose(-1, -2)) * scaling
    n = q.shape[2]
    i = torch.arange(n, device=q.device)
    ok = i[None, :] <= i[:, None]
    if sliding_window:
        ok = ok & ((i[:, None] - i[None, :]) < sliding_window)
    p = torch.softmax(s.masked_fill(~ok, float("-inf")), -1)
    return (p @ vv).to(q.dtype).transpose(1, 2).contiguous(), None


def small_cfg(impl):
    return Gemma4SyntheticConfig(vocab_size=500, hidden_size=128, num_layers=5, global_heads=4, global_kv_heads=1,
                                 global_head_dim=64, local_heads=2, local_kv_heads=1, local_head_dim=32,
                                 sliding_window=16, intermediate_size=256, attn_implementation=impl)


def test_layer_pattern_and_hf_calling_convention():
    ALL_ATTENTION_FUNCTIONS["explicit_test"] = explicit_attention
    CALLS.clear()
    model = Gemma4SyntheticDecoder(small_cfg("explicit_test")).init_weights(seed=1)
    ids = torch.randint(0, 500, (2, 40), generator=torch.Generator().manual_seed(0))
    logits = model(ids)
    assert logits.shape == (2, 40, 500) and torch.isfinite(logits).all()
    assert len(CALLS) == 5
    # layer 4 (every 5th) is global, the others sliding
    assert [c[3] for c in CALLS] == [16, 16, 16, 16, None]
    assert CALLS[4][0] == (2, 4, 40, 64) and CALLS[0][1] == (2, 1, 40, 32)
    assert not any(c[4] for c in CALLS), "q arrives as a (B, N, H, D) view, as in transformers"


def test_full_config_shapes():
    cfg = Gemma4SyntheticConfig()
    globals_ = [i for i in range(cfg.num_layers) if cfg.is_global(i)]
    assert globals_ == [4, 9, 14, 19, 24, 29, 34]
