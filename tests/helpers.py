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
# (name, criterion, max_abs vs fp32, cosine) of every assert_close call; written
# to $GQAFA_PARITY_REPORT at the end of the session when that is set.
REPORT = []

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


def torch_ref(q, k, v, do, causal, slide, scale=None, chunk=1024, need_grad=True, emulate=False,
              magnitudes=False):
    """fp32 forward (O, LSE) and backward (dQ, dK, dV) of the same math as the
    oracle, chunked over query rows; runs on q's device.

    emulate=True applies the 16-bit roundings the reference algorithm itself
    performs (P cast to the input dtype before P.V and P^T.dO, attention.py:373
    and :1194; dS cast before dS.K and dS^T.Q, :791 and :1200; O stored in the
    input dtype before delta = rowsum(dO*O)), everything else in fp32.

    magnitudes=True returns instead the absolute-value products |P||V|, 0,
    scale|dS||K|, scale|dS^T||Q|, |P^T||dO| whose entries bound, to first
    order in the unit roundoff u, how far rounding P and dS to 16 bits can move
    each output element (|error| <= u * magnitude)."""
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
        rnd = (lambda t: t.to(q.dtype).float()) if emulate else (lambda t: t)
        if magnitudes:
            ab = torch.abs
            o[:, :, q0:q1] = p @ ab(vv)
            lse[:, :, q0:q1] = 0
            doi = do32[:, :, q0:q1]
            o_true = p @ vv
            ds = p * ((doi @ vv.transpose(-1, -2)) - (doi * o_true).sum(-1, keepdim=True))
            dq[:, :, q0:q1] = (ab(ds) @ ab(kk)) * scale
            dkk += (ab(ds).transpose(-1, -2) @ ab(q32[:, :, q0:q1])) * scale
            dvv += p.transpose(-1, -2) @ ab(doi)
            continue
        o[:, :, q0:q1] = rnd(p) @ vv
        lse[:, :, q0:q1] = l
        if need_grad:
            doi = do32[:, :, q0:q1]
            delta = (doi * rnd(o[:, :, q0:q1])).sum(-1, keepdim=True)
            dp = doi @ vv.transpose(-1, -2)
            ds = rnd(p * (dp - delta))
            dq[:, :, q0:q1] = (ds @ kk) * scale
            dkk += (ds.transpose(-1, -2) @ q32[:, :, q0:q1]) * scale
            dvv += rnd(p).transpose(-1, -2) @ doi
    if not need_grad:
        return o, lse
    Hkv = k.shape[1]
    dk = dkk.view(B, Hkv, G, N, D).sum(2)
    dv = dvv.view(B, Hkv, G, N, D).sum(2)
    return o, lse, dq, dk, dv


def metrics(x, ref):
    """(max-abs difference, cosine similarity), in float64 on x's device."""
    x = x.detach().reshape(-1).double()
    r = ref.detach().to(x.device).reshape(-1).double()
    max_abs = (x - r).abs().max().item() if x.numel() else 0.0
    denom = (x.norm() * r.norm()).item()
    cos = (x @ r).item() / denom if denom > 0 else 1.0
    return max_abs, cos


def half_ulp(ref: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Half a unit in the last place of `dtype` at the magnitude of `ref`."""
    mant_bits = {torch.bfloat16: 7, torch.float16: 10}[dtype]
    _, e = torch.frexp(ref.abs().float())
    return torch.ldexp(torch.ones_like(ref, dtype=torch.float32), e - 2 - mant_bits)


UNIT_ROUNDOFF = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def assert_close(name, x, ref, atol=ATOL, cos_min=COS_MIN, emulated=None, magnitude=None):
    """Parity check of a 16-bit kernel output against an fp32 computation.

    Passes on the first of these that holds (the message names which):
      A. north-star criterion: max-abs <= atol and cosine >= cos_min;
      B. the same except for storage rounding: every element within
         atol + half_ulp(dtype, |ref|) (an output of magnitude m must be stored
         with up to half an ulp(m) of error: 0.031 for bf16 at |m| in [8, 16));
      C. B against `emulated`, the fp32 computation that applies the 16-bit
         roundings of P and dS the reference algorithm itself performs;
      D. every element within atol + half_ulp + 2u * magnitude, the
         first-order error bound of those roundings (u = unit roundoff of the
         dtype, magnitude from torch_ref(..., magnitudes=True)); this is what
         limits gradients summed over many GQA heads of N(0,1) inputs.
    Cosine is only meaningful when the reference is not numerically zero
    (e.g. dQ of a one-token sequence); then max-abs <= atol alone applies.
    """
    assert torch.isfinite(x.float()).all(), f"{name}: non-finite values"
    xf = x.detach().float()
    rf = ref.detach().float().to(xf.device)
    max_abs, cos = metrics(xf, rf)
    negligible = rf.abs().max().item() < 1e-3
    if negligible:
        assert max_abs <= atol, f"{name}: max_abs={max_abs:.3e} on a ~zero reference"
        REPORT.append((name, "A0", max_abs, cos))
        return "A", max_abs, cos
    if max_abs <= atol and cos >= cos_min:
        REPORT.append((name, "A", max_abs, cos))
        return "A", max_abs, cos
    msgs = [f"A: max_abs={max_abs:.3e} cos={cos:.6f}"]
    if x.dtype in (torch.bfloat16, torch.float16):
        excess = ((xf - rf).abs() - half_ulp(rf, x.dtype)).max().item()
        if excess <= atol and cos >= cos_min:
            REPORT.append((name, "B", max_abs, cos))
            return "B", max_abs, cos
        msgs.append(f"B: excess over storage rounding {excess:.3e}")
        if emulated is not None:
            ef = emulated.detach().float().to(xf.device)
            e_abs, e_cos = metrics(xf, ef)
            e_excess = ((xf - ef).abs() - half_ulp(ef, x.dtype)).max().item()
            if e_excess <= atol and e_cos >= cos_min and cos >= cos_min:
                REPORT.append((name, "C", max_abs, cos))
                return "C", max_abs, cos
            msgs.append(f"C: vs rounding-emulated fp32 max_abs={e_abs:.3e} excess={e_excess:.3e} cos={e_cos:.6f}")
        if magnitude is not None:
            mf = magnitude.detach().float().to(xf.device)
            bound = atol + half_ulp(rf, x.dtype) + 2 * UNIT_ROUNDOFF[x.dtype] * mf
            worst = ((xf - rf).abs() - bound).max().item()
            if worst <= 0 and cos >= cos_min:
                REPORT.append((name, "D", max_abs, cos))
                return "D", max_abs, cos
            msgs.append(f"D: exceeds the rounding bound by {worst:.3e}")
    raise AssertionError(f"{name}: " + "; ".join(msgs) + f"; bound {atol}, cos >= {cos_min}, "
                         f"max|ref|={rf.abs().max().item():.3g}")
