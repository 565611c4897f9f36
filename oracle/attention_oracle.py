"""CPU oracle for the GQA flash-attention path. TEST INFRASTRUCTURE ONLY.

This module is the parity checker: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it. The product path
(gemma_triton_flash_attn) never calls it and has no CPU fallback.

It restates, in numpy, the arithmetic of the reference
zzhhjjj/gemma-triton-flash-attn for the path its kernels compute:

  forward   flash_attn/attention.py:244-388  (_flash_attn_gqa_kernel)
            O = softmax(scale * Q K^T + mask) V, per query head h using KV head
            h // (H_Q // H_KV) (attention.py:272); the mask is k <= q (causal)
            and additionally q - k < W (sliding window, only with causal,
            attention.py:347-356); LSE = natural-log logsumexp of the scaled,
            masked scores (attention.py:384-388).
  backward  flash_attn/attention.py:686-797 and :1079-1213
            delta = rowsum(dO * O)                       (:738-742)
            P = exp(scale * S - LSE)                     (:776-779)
            dP = dO V^T, dS = P * (dP - delta)           (:781-784, :1188-1197)
            dQ = scale * dS K, dK = scale * sum_g dS^T Q, dV = sum_g P^T dO
            (:793, :1202; the packed kernel sums over the G query heads of a group)
  window    slide_size >= N means plain causal (:1442-1443).

The oracle is pinned against the reference itself: tests/golden/make_golden.py
imports the reference's eager functions attention_gqa_ref / attention_swa_ref
(attention.py:611-642, SDPA in fp32) and differentiates them with autograd;
tests/test_oracle.py checks this module against those fixtures.

Computation is float32 by default (the "fp32 computation" of the parity
criterion) or float64, chunked over query rows so large N stays in memory.
"""
from __future__ import annotations

import numpy as np

__all__ = ["attention_fwd", "attention_bwd", "mask_block", "attended_pairs", "attn_flops"]


def _window(causal: bool, window: int, n: int) -> int:
    if not causal or window is None or window <= 0 or window >= n:
        return 0
    return int(window)


def mask_block(q0: int, q1: int, k0: int, k1: int, n: int, causal: bool, window: int) -> np.ndarray:
    """Boolean (q1-q0, k1-k0) mask: True where query q attends key k."""
    q = np.arange(q0, q1)[:, None]
    k = np.arange(k0, k1)[None, :]
    ok = (q < n) & (k < n)
    if causal:
        ok = ok & (k <= q)
        if window:
            ok = ok & ((q - k) < window)
    return ok


def attention_fwd(q, k, v, causal=False, window=0, scale=None, dtype=np.float32, chunk=512, q_offset=0):
    """Returns (O, LSE). q: (B,Hq,Nq,D), k/v: (B,Hkv,N,D) arrays of any float type.

    The query rows are sequence positions q_offset .. q_offset+Nq-1 (Nq = N and
    q_offset = 0 for full self-attention; a row subset for bounded samples).
    """
    b_sz, hq, n_q, d = q.shape
    n = k.shape[2]
    hkv = k.shape[1]
    g = hq // hkv
    w = _window(causal, window, n)
    scale = (1.0 / np.sqrt(d)) if scale is None else scale
    o = np.zeros((b_sz, hq, n_q, d), dtype=dtype)
    lse = np.full((b_sz, hq, n_q), -np.inf, dtype=dtype)
    for b in range(b_sz):
        for h in range(hq):
            kh = k[b, h // g].astype(dtype)
            vh = v[b, h // g].astype(dtype)
            for q0 in range(0, n_q, chunk):
                q1 = min(n_q, q0 + chunk)
                a0, a1 = q0 + q_offset, q1 + q_offset
                k0 = max(0, a0 - w + 1) if w else 0
                k1 = min(n, a1) if causal else n
                s = (q[b, h, q0:q1].astype(dtype) @ kh[k0:k1].T) * dtype(scale)
                m = mask_block(a0, a1, k0, k1, n, causal, w)
                s = np.where(m, s, -np.inf)
                mx = s.max(axis=1, keepdims=True)
                mx = np.where(np.isfinite(mx), mx, 0)
                p = np.exp(s - mx)
                l = p.sum(axis=1, keepdims=True)
                o[b, h, q0:q1] = (p / np.where(l > 0, l, 1)) @ vh[k0:k1]
                lse[b, h, q0:q1] = np.where(l[:, 0] > 0, mx[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1)), -np.inf)
    return o, lse


def attention_bwd(q, k, v, o, lse, do, causal=False, window=0, scale=None, dtype=np.float32, chunk=512,
                  q_offset=0):
    """Returns (dQ, dK, dV, delta) given the forward's O and LSE (query rows as
    in attention_fwd; dK/dV then hold the contributions of those rows only)."""
    b_sz, hq, n_q, d = q.shape
    n = k.shape[2]
    hkv = k.shape[1]
    g = hq // hkv
    w = _window(causal, window, n)
    scale = (1.0 / np.sqrt(d)) if scale is None else scale
    dq = np.zeros((b_sz, hq, n_q, d), dtype=dtype)
    dk = np.zeros((b_sz, hkv, n, d), dtype=dtype)
    dv = np.zeros((b_sz, hkv, n, d), dtype=dtype)
    delta = (do.astype(dtype) * o.astype(dtype)).sum(axis=-1)
    for b in range(b_sz):
        for h in range(hq):
            kv = h // g
            kh = k[b, kv].astype(dtype)
            vh = v[b, kv].astype(dtype)
            for q0 in range(0, n_q, chunk):
                q1 = min(n_q, q0 + chunk)
                a0, a1 = q0 + q_offset, q1 + q_offset
                k0 = max(0, a0 - w + 1) if w else 0
                k1 = min(n, a1) if causal else n
                qh = q[b, h, q0:q1].astype(dtype)
                doh = do[b, h, q0:q1].astype(dtype)
                s = (qh @ kh[k0:k1].T) * dtype(scale)
                m = mask_block(a0, a1, k0, k1, n, causal, w)
                p = np.where(m, np.exp(s - lse[b, h, q0:q1, None].astype(dtype)), 0)
                dp = doh @ vh[k0:k1].T
                ds = p * (dp - delta[b, h, q0:q1, None])
                dq[b, h, q0:q1] = (ds @ kh[k0:k1]) * dtype(scale)
                dk[b, kv, k0:k1] += (ds.T @ qh) * dtype(scale)
                dv[b, kv, k0:k1] += p.T @ doh
    return dq, dk, dv, delta


def attended_pairs(n: int, causal: bool, window: int = 0) -> int:
    """Number of (q, k) pairs a head attends: the FLOP basis of the benchmarks.

    Causal is charged as N^2/2 (the reference's convention,
    benchmarks/run_final_benchmark.py:217-224); sliding window W < N as
    N*W - W(W-1)/2; non-causal as N^2.
    """
    w = _window(causal, window, n)
    if not causal:
        return n * n
    if w:
        return n * w - w * (w - 1) // 2
    return n * n // 2


def attn_flops(b: int, hq: int, n: int, d: int, causal: bool, window: int = 0, bwd: bool = False) -> int:
    """fwd = 4*B*H_Q*D*P, fwd+bwd = 14*B*H_Q*D*P (= 2 and 7 * B*H*N^2*D for causal)."""
    pairs = attended_pairs(n, causal, window)
    return (14 if bwd else 4) * b * hq * d * pairs
