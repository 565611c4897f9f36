"""The reference's eager CPU attention path, restated. TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs (``cpu_baseline`` and ``--impl
reference``) may import this module. The product path never does.

The reference's one CPU-capable implementation of the attention math is its
eager helper ``attention_gqa_ref(q, k, v, causal)``
(flash_attn/attention.py:611-619). It repeats every KV head to the query head
count (``repeat_interleave`` along dim 1) and calls
``torch.nn.functional.scaled_dot_product_attention`` with ``is_causal``; the
backward is torch autograd through that call. ``sdpa_gqa`` below performs the
same two torch operations in the same order, so on the same fp32 CPU
tensors it runs the same ATen kernels as the reference function. The
sliding-window variant follows ``attention_swa_ref`` (attention.py:622-642):
a boolean (N, N) mask, key j visible to query i iff j <= i and i - j < W.

``tests/test_oracle.py`` checks this restatement bit-exactly against the
reference module when a checkout is available, and against the committed
golden fixtures (which the reference produced) otherwise.
"""
from __future__ import annotations

import os
import statistics
import time

import torch

__all__ = ["sdpa_gqa", "time_fwd_bwd", "use_all_cores"]


def sdpa_gqa(q, k, v, causal=False, window=0):
    """O for (B, H_Q, N, D) q and (B, H_KV, N, D) k, v; scale 1/sqrt(D)."""
    g = q.shape[1] // k.shape[1]
    if g != 1:
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
    n = q.shape[2]
    if causal and window and 0 < window < n:
        i = torch.arange(n)
        allowed = (i[None, :] <= i[:, None]) & ((i[:, None] - i[None, :]) < window)
        return torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=allowed)
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=bool(causal))


def use_all_cores():
    """Give torch's intra-op pool every host core (torchrun sets OMP_NUM_THREADS=1)
    and return the thread count actually in use."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:  # the BLAS pool, when threadpoolctl can reach it
        from threadpoolctl import threadpool_limits

        threadpool_limits(n)
    except Exception:
        pass
    return torch.get_num_threads()


def time_fwd_bwd(q, k, v, do, causal, window=0, warmup=3, reps=9, fwd_only=False):
    """Median seconds of one forward (+ backward via autograd) of sdpa_gqa."""
    qq, kk, vv = (t.detach().clone().requires_grad_(not fwd_only) for t in (q, k, v))

    def run():
        if fwd_only:
            with torch.no_grad():
                sdpa_gqa(qq, kk, vv, causal, window)
            return
        qq.grad = kk.grad = vv.grad = None
        o = sdpa_gqa(qq, kk, vv, causal, window)
        o.backward(do)

    for _ in range(warmup):
        run()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return statistics.median(times)
