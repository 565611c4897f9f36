"""FLOP accounting of the benchmarks (the reference's convention).

Charged work per query head: fwd = 4*D*P and fwd+bwd = 14*D*P, where P is the
number of attended (query, key) pairs. Causal attention is charged N^2/2 pairs
(so fwd = 2*B*H*N^2*D and fwd+bwd = 7*B*H*N^2*D, as in the reference's
benchmarks/run_final_benchmark.py:217-224); a causal sliding window W < N is
window-limited, P = N*W - W(W-1)/2; non-causal is N^2.
"""
from __future__ import annotations

__all__ = ["attended_pairs", "attn_flops", "kernel_flops"]


def attended_pairs(n: int, causal: bool, window: int = 0) -> int:
    if not causal:
        return n * n
    if window and 0 < window < n:
        return n * window - window * (window - 1) // 2
    return n * n // 2


def attn_flops(b: int, hq: int, n: int, d: int, causal: bool, window: int = 0, bwd: bool = False) -> int:
    return (14 if bwd else 4) * b * hq * d * attended_pairs(n, causal, window)


# GEMMs (each 2*D*P FLOPs per query head) that each kernel's own math needs:
# fwd Q.K^T and P.V; dQ recomputes Q.K^T, forms dO.V^T and dS.K; dK the same
# two scores plus dS^T.Q; dV recomputes Q.K^T and forms P^T.dO. The
# materialised backward's dQ kernel ("dqps") does the dQ kernel's three and
# stores P and dS; its dK/dV kernel ("dkv") forms dS^T.Q and P^T.dO only.
KERNEL_GEMMS = {"fwd": 2, "dq": 3, "dk": 3, "dv": 2, "dqps": 3, "dkv": 2}


def kernel_flops(kernel: str, b: int, hq: int, n: int, d: int, causal: bool, window: int = 0) -> int:
    return KERNEL_GEMMS[kernel] * 2 * b * hq * d * attended_pairs(n, causal, window)
