"""Forward with a KV cache longer than the queries (decode and chunked
prefill), through attention_flash_gqa / gqafa_fwd_kv and the HF adapter,
against an fp32 computation: with causal attention query row r sits at key
position r + N_k - N_q; a window counts back from there; without causal every
query sees every key. The reference takes the key length from q and reads a
wrong key range here (flash_attn/attention.py:552-553), so this is checked
against the math, not against the reference's behaviour."""
import math
import types

import pytest
import torch

import gemma_triton_flash_attn as gfa
from gemma_triton_flash_attn import _lib
from gemma_triton_flash_attn.attention import flash_attn_gqa_forward_with_lse
from helpers import LSE_ATOL, assert_close, seeded

pytestmark = pytest.mark.gpu
DEV = "cuda"


def kv_ref(q, k, v, causal, window, scale=None):
    B, Hq, Nq, D = q.shape
    Nk = k.shape[2]
    G = Hq // k.shape[1]
    scale = 1 / math.sqrt(D) if scale is None else scale
    kk = k.float().repeat_interleave(G, 1)
    vv = v.float().repeat_interleave(G, 1)
    s = (q.float() @ kk.transpose(-1, -2)) * scale
    pos = torch.arange(Nq, device=q.device)[:, None] + (Nk - Nq)
    key = torch.arange(Nk, device=q.device)[None, :]
    ok = torch.ones(Nq, Nk, dtype=torch.bool, device=q.device)
    if causal:
        ok = key <= pos
        if window and 0 < window < Nk:
            ok = ok & (pos - key < window)
    s = s.masked_fill(~ok, float("-inf"))
    lse = torch.logsumexp(s, -1)
    return torch.softmax(s, -1) @ vv, lse


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert _lib.device_status(torch.cuda.current_device(), reset=True) == 0, "a kernel wait timed out"


CASES = [
    # (B, Hq, Hkv, Nq, Nk, causal, window)
    (2, 8, 2, 1, 1000, True, 0),        # one decode step
    (1, 32, 4, 1, 4097, True, 0),
    (1, 16, 8, 1, 3000, True, 512),     # sliding-window layer, cache past the window
    (1, 4, 1, 7, 300, True, 0),
    (1, 8, 2, 128, 700, True, 0),       # chunked prefill
    (2, 4, 2, 300, 1500, True, 200),
    (1, 4, 2, 130, 130, True, 0),       # N_k == N_q through the same entry
    (1, 4, 4, 64, 1000, False, 0),      # non-causal cross attention
    (1, 8, 2, 200, 90, False, 0),       # non-causal, fewer keys than queries
]


@pytest.mark.parametrize("D", [64, 128, 256, 512])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_H{}-{}_Nq{}_Nk{}_c{}_w{}".format(*c))
def test_kv_cache_forward_matches_fp32(case, D):
    B, Hq, Hkv, Nq, Nk, causal, window = case
    dt = torch.bfloat16 if D in (128, 512) else torch.float16
    q = seeded((B, Hq, Nq, D), Nq + D, 1.0, dt, DEV)
    k = seeded((B, Hkv, Nk, D), Nk + D + 1, 1.0, dt, DEV)
    v = seeded((B, Hkv, Nk, D), Nk + D + 2, 1.0, dt, DEV)
    o, lse = flash_attn_gqa_forward_with_lse(q, k, v, causal, window)
    inf = gfa.attention_flash_gqa(q, k, v, causal=causal, slide_size=window)
    torch.cuda.synchronize()
    ro, rl = kv_ref(q, k, v, causal, window)
    assert torch.equal(o, inf)
    assert_close(f"kv D{D} {case} O", o, ro)
    assert (lse - rl).abs().max().item() <= LSE_ATOL


def test_kv_cache_validation():
    q = torch.zeros(1, 4, 100, 256, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(1, 2, 50, 256, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="key length"):
        gfa.attention_flash_gqa(q, k, k, causal=True)
    with pytest.raises(ValueError, match="self-attention"):
        gfa.flash_attn_gqa_train(q, k, k, causal=False)


def test_hf_adapter_decode_step():
    """The adapter under no_grad with a cache longer than the query (what
    generate() does) runs the KV-cache forward and returns (B, N, H, D)."""
    B, Hq, Hkv, Nk, D = 1, 16, 8, 777, 256
    q = seeded((B, Hq, 1, D), 1, 1.0, torch.bfloat16, DEV)
    k = seeded((B, Hkv, Nk, D), 2, 1.0, torch.bfloat16, DEV)
    v = seeded((B, Hkv, Nk, D), 3, 1.0, torch.bfloat16, DEV)
    module = types.SimpleNamespace(head_dim=D, is_causal=True)
    with torch.no_grad():
        out, w = gfa.triton_gqa_attention(module, q, k, v, None, scaling=1.0, sliding_window=512)
    assert w is None and out.shape == (B, 1, Hq, D)
    ro, _ = kv_ref(q, k, v, True, 512, scale=1.0)
    assert_close("adapter decode", out.transpose(1, 2), ro)
    qg = q.clone().requires_grad_(True)
    with pytest.raises(NotImplementedError):
        gfa.triton_gqa_attention(module, qg, k, v, None, scaling=1.0)
