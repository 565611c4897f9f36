"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own eager implementation of the attention math —
``attention_gqa_ref`` (flash_attn/attention.py:611-619) and
``attention_swa_ref`` (flash_attn/attention.py:622-642), both SDPA in fp32 on
CPU — imported from a checkout of zzhhjjj/gemma-triton-flash-attn, and
differentiates it with autograd for dQ/dK/dV. The reference returns no LSE;
it is computed here with the kernel's documented convention (natural log of
the scaled, masked scores, flash_attn/attention.py:384-388) directly with
torch.logsumexp, independently of oracle/.

Usage (needs the reference checkout; the fixtures are committed, so the GPU
box and the CPU tests never run this):

    python tests/golden/make_golden.py /path/to/gemma-triton-flash-attn

Inputs are drawn N(0,1) * factor from seeded torch.Generator streams, rounded
to the case's 16-bit dtype (the kernels' input type), and stored as raw 16-bit
patterns; outputs are stored as float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, H_Q, H_KV, N, D, causal, slide_size, dtype, input factor)
CASES = [
    ("gqa4_causal_d32", 1, 4, 1, 50, 32, True, 0, "bf16", 1.0),
    ("mha_noncausal_d16", 2, 3, 3, 37, 16, False, 0, "fp16", 1.0),
    ("gqa2_swa8_d64", 1, 4, 2, 61, 64, True, 8, "fp16", 1.0),
    ("gqa8_swa_ge_n_d32", 1, 8, 1, 24, 32, True, 64, "bf16", 0.5),
    ("noncausal_window_ignored", 1, 2, 1, 29, 32, False, 5, "bf16", 1.0),
    ("kernel_d256_swa24", 1, 2, 1, 72, 256, True, 24, "bf16", 1.0),
    ("kernel_d512_causal", 1, 2, 1, 40, 512, True, 0, "fp16", 0.5),
]

_TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _inputs(b, hq, hkv, n, d, dt, factor, seed):
    shapes = [(b, hq, n, d), (b, hkv, n, d), (b, hkv, n, d), (b, hq, n, d)]
    out = []
    for i, shp in enumerate(shapes):
        g = torch.Generator().manual_seed(seed + i)
        x = torch.randn(shp, generator=g, dtype=torch.float32) * factor
        out.append(x.to(_TORCH_DT[dt]))
    return out  # q, k, v, do (16-bit)


def _lse(q, k, causal, slide):
    b, hq, n, d = q.shape
    g = hq // k.shape[1]
    kk = k.repeat_interleave(g, dim=1)
    s = (q @ kk.transpose(-1, -2)) / (d ** 0.5)
    i = torch.arange(n)
    ok = torch.ones(n, n, dtype=torch.bool)
    if causal:
        ok = i[None, :] <= i[:, None]
        if 0 < slide < n:
            ok = ok & ((i[:, None] - i[None, :]) < slide)
    s = s.masked_fill(~ok, float("-inf"))
    return torch.logsumexp(s, dim=-1)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from flash_attn.attention import attention_gqa_ref, attention_swa_ref  # noqa: E402

    for ci, (name, b, hq, hkv, n, d, causal, slide, dt, fac) in enumerate(CASES):
        q16, k16, v16, do16 = _inputs(b, hq, hkv, n, d, dt, fac, seed=1000 + 10 * ci)
        q, k, v, do = (t.float().requires_grad_(i < 3) for i, t in enumerate((q16, k16, v16, do16)))
        if causal and 0 < slide < n:
            o = attention_swa_ref(q, k, v, slide)
        else:
            o = attention_gqa_ref(q, k, v, causal=causal)
        o.backward(do)
        lse = _lse(q.detach(), k.detach(), causal, slide)
        bits = lambda t: t.view(torch.int16).numpy().copy()  # noqa: E731
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([b, hq, hkv, n, d, int(causal), slide], dtype=np.int64),
            dtype=np.array(dt),
            q=bits(q16), k=bits(k16), v=bits(v16), do=bits(do16),
            o=o.detach().numpy(), lse=lse.numpy(),
            dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy(),
        )
        print("wrote", name)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
