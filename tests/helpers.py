"""Shared test utilities: seeded inputs, fixture loading, error metrics and an
fp32 PyTorch reference of the attention math (usable on GPU for sizes the
numpy oracle would take too long on)."""
from __future__ import annotations

import glob
import math
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {"bf16": torch.bfloat16, "fp16": torch.float16}

# Parity criteria: outputs and gradients within max-abs
# 2e-2 and fp32 cosine >= 0.9999 of an fp32 computation; LSE within 1e-3.
ATOL = 2e-2
COS_MIN = 0.9999
LSE_ATOL = 1e-3


def golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(path):
    z = np.load(path)
    b, hq, hkv, n, d, causal, slide = (int(x) for x in z["meta"])
    dt = str(z["dtype"])
    tdt = DT[dt]

    def t16(a):
        return torch.from_numpy(a.copy()).view(tdt)

    case = dict(B=b, Hq=hq, Hkv=hkv, N=n, D=d, causal=bool(causal), slide=slide, dtype=dt,
                q=t16(z["q"]), k=t16(z["k"]), v=t16(z["v"]), do=t16(z["do"]))
    for key in ("o", "lse", "dq", "dk", "dv"):
        case[key] = torch.from_numpy(z[key].copy())
    return case


def seeded(shape, seed, factor=1.0, dtype=torch.bfloat16, device="cpu"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(shape, generator=g, dtype=torch.float32) * factor
    return x.to(dtype).to(device)


def make_inputs(B, Hq, Hkv, N, D, dtype=torch.bfloat16, factor=1.0, seed=0, device="cpu"):
    q = seeded((B, Hq, N, D), seed, factor, dtype, device)
    k = seeded((B, Hkv, N, D), seed + 1, factor, dtype, device)
    v = seeded((B, Hkv, N, D), seed + 2, factor, dtype, device)
    do = seeded((B, Hq, N, D), seed + 3, factor, dtype, device)
    return q, k, v, do


def torch_ref(q, k, v, do, causal, slide, scale=None, chunk=1024, need_grad=True):
    """fp32 forward (O, LSE) and backward (dQ, dK, dV) of the same math as the
    oracle, chunked over query rows; runs on q's device."""
    q32, k32, v32 = q.float(), k.float(), v.float()
    B, Hq, N, D = q.shape
    G = Hq // k.shape[1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    w = slide if (causal and 0 < slide < N) else 0
    kk = k32.repeat_interleave(G, dim=1)
    vv = v32.repeat_interleave(G, dim=1)
    o = torch.empty_like(q32)
    lse = torch.empty(B, Hq, N, device=q.device)
    dq = torch.zeros_like(q32)
    dkk = torch.zeros_like(kk)
    dvv = torch.zeros_like(vv)
    do32 = do.float() if do is not None else None
    idx = torch.arange(N, device=q.device)
    for q0 in range(0, N, chunk):
        q1 = min(N, q0 + chunk)
        qi = idx[q0:q1, None]
        ok = torch.ones(q1 - q0, N, dtype=torch.bool, device=q.device)
        if causal:
            ok = idx[None, :] <= qi
            if w:
                ok = ok & ((qi - idx[None, :]) < w)
        s = (q32[:, :, q0:q1] @ kk.transpose(-1, -2)) * scale
        s = s.masked_fill(~ok, float("-inf"))
        l = torch.logsumexp(s, dim=-1)
        p = torch.exp(s - l[..., None])
        o[:, :, q0:q1] = p @ vv
        lse[:, :, q0:q1] = l
        if need_grad:
            doi = do32[:, :, q0:q1]
            delta = (doi * o[:, :, q0:q1]).sum(-1, keepdim=True)
            dp = doi @ vv.transpose(-1, -2)
            ds = p * (dp - delta)
            dq[:, :, q0:q1] = (ds @ kk) * scale
            dkk += (ds.transpose(-1, -2) @ q32[:, :, q0:q1]) * scale
            dvv += p.transpose(-1, -2) @ doi
    if not need_grad:
        return o, lse
    Hkv = k.shape[1]
    dk = dkk.view(B, Hkv, G, N, D).sum(2)
    dv = dvv.view(B, Hkv, G, N, D).sum(2)
    return o, lse, dq, dk, dv


def metrics(x, ref):
    x = x.detach().float().cpu().reshape(-1).double()
    r = ref.detach().float().cpu().reshape(-1).double()
    max_abs = (x - r).abs().max().item() if x.numel() else 0.0
    denom = (x.norm() * r.norm()).item()
    cos = (x @ r).item() / denom if denom > 0 else 1.0
    return max_abs, cos


def assert_close(name, x, ref, atol=ATOL, cos_min=COS_MIN):
    assert torch.isfinite(x.float()).all(), f"{name}: non-finite values"
    max_abs, cos = metrics(x, ref)
    assert max_abs <= atol and cos >= cos_min, f"{name}: max_abs={max_abs:.3e} (<= {atol}), cos={cos:.6f} (>= {cos_min})"
    return max_abs, cos
