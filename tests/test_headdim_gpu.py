"""head_dim 64 and 128 (the reference accepts any power of two up to 512,
docs/api.md:63, and publishes a head_dim-128 number, README.md:26): the 1-CTA
kernels with the recomputing backward, through the public API, against the
fp32 reference on causal, sliding-window, non-causal, ragged and GQA shapes."""
import pytest
import torch

import gemma_triton_flash_attn as gfa
from gemma_triton_flash_attn import _lib
from gemma_triton_flash_attn.attention import bwd_workspace_size, flash_attn_gqa_backward, \
    flash_attn_gqa_forward_with_lse
from helpers import LSE_ATOL, assert_close, make_inputs, torch_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [
    # (B, Hq, Hkv, N, causal, window)
    (1, 4, 1, 1, True, 0),
    (1, 4, 2, 300, True, 0),
    (2, 8, 2, 777, True, 0),
    (1, 2, 2, 129, False, 0),
    (1, 8, 4, 1000, True, 128),
    (1, 4, 1, 96, True, 95),
    (2, 16, 1, 257, True, 0),
    (1, 16, 8, 4096, True, 1024),
]


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert _lib.device_status(torch.cuda.current_device(), reset=True) == 0, "a kernel wait timed out"


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_H{}-{}_N{}_c{}_w{}".format(*c))
def test_small_head_dims_match_fp32(case, D, dt):
    B, Hq, Hkv, N, causal, window = case
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, 1.0, seed=N + D, device=DEV)
    o, lse = flash_attn_gqa_forward_with_lse(q, k, v, causal, window)
    dq, dk, dv = flash_attn_gqa_backward(q, k, v, o, lse, do, causal, window)
    torch.cuda.synchronize()
    ref = torch_ref(q, k, v, do, causal, window)
    emu = torch_ref(q, k, v, do, causal, window, emulate=True)
    mag = torch_ref(q, k, v, do, causal, window, magnitudes=True)
    assert (lse - ref[1]).abs().max().item() <= LSE_ATOL
    for i, (name, x) in enumerate((("O", o), ("LSE", None), ("dQ", dq), ("dK", dk), ("dV", dv))):
        if x is not None:
            assert_close(f"D{D} {case} {name}", x, ref[i], emulated=emu[i], magnitude=mag[i])


@pytest.mark.parametrize("D", [64, 128])
def test_small_head_dims_autograd_and_inference(D):
    q, k, v, do = make_inputs(2, 8, 2, 640, D, torch.bfloat16, 0.5, seed=3, device=DEV)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    out = gfa.flash_attn_gqa_train(qg, kg, vg, causal=True, slide_size=200)
    out.backward(do)
    inf = gfa.attention_flash_gqa(q, k, v, causal=True, slide_size=200)
    assert torch.equal(out.detach(), inf)
    ref = torch_ref(q, k, v, do, True, 200)
    for name, x, r in (("O", out, ref[0]), ("dQ", qg.grad, ref[2]), ("dK", kg.grad, ref[3]), ("dV", vg.grad, ref[4])):
        assert_close(f"autograd D{D} {name}", x, r)
    # no workspace at these head dims: the backward recomputes
    assert bwd_workspace_size(2, 8, 2, 640, D, True, 200) == 0
