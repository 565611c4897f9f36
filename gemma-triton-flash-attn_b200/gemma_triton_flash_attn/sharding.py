"""Multi-GPU sharding of the attention path over (batch, KV-head group) units.

Every (b, kv_head) pair is an independent unit in both passes: its G query
heads read only that KV head, and dK/dV of the KV head depend only on those G
query heads (the packed-GQA reduction of the reference's dK/dV kernel,
flash_attn/attention.py:1079-1213). Each rank therefore computes whole units
with no communication inside the kernels; ``torch.distributed`` all-gathers
(NCCL over NVLink on GPUs, gloo in the CPU tests) reassemble the outputs.

Units are assigned in contiguous, balanced blocks of the flattened index
``u = b * H_KV + kv_head``. Inputs are replicated on every rank; each rank
slices its units as strided views (no copies: the C ABI takes strides).

The per-unit compute is injectable (``fwd_fn`` / ``bwd_fn``) so the
partitioning and reassembly logic can be exercised on CPU ranks with a
stand-in; by default it is the CUDA kernel path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["ShardPlan", "sharded_forward", "sharded_backward"]


@dataclass(frozen=True)
class ShardPlan:
    batch: int
    heads_q: int
    heads_kv: int
    world: int
    rank: int

    @property
    def num_units(self) -> int:
        return self.batch * self.heads_kv

    @property
    def group(self) -> int:
        return self.heads_q // self.heads_kv

    def unit_range(self, rank: int | None = None) -> tuple[int, int]:
        """[u0, u1) for `rank`: balanced contiguous blocks (first ranks get the extra)."""
        r = self.rank if rank is None else rank
        base, extra = divmod(self.num_units, self.world)
        u0 = r * base + min(r, extra)
        return u0, u0 + base + (1 if r < extra else 0)

    @property
    def max_units(self) -> int:
        return -(-self.num_units // self.world)

    def runs(self, rank: int | None = None):
        """Contiguous KV-head runs of a rank's units: (b, kv0, kv1) triples."""
        u0, u1 = self.unit_range(rank)
        u = u0
        while u < u1:
            b, kv0 = divmod(u, self.heads_kv)
            kv1 = min(self.heads_kv, kv0 + (u1 - u))
            yield b, kv0, kv1
            u += kv1 - kv0


def _default_fwd(q, k, v, causal, slide_size, softmax_scale):
    from .attention import flash_attn_gqa_forward_with_lse

    return flash_attn_gqa_forward_with_lse(q, k, v, causal, slide_size, softmax_scale)


def _default_bwd(q, k, v, o, lse, do, causal, slide_size, softmax_scale):
    from .attention import flash_attn_gqa_backward

    return flash_attn_gqa_backward(q, k, v, o, lse, do, causal, slide_size, softmax_scale)


def _gather_units(plan: ShardPlan, local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-unit blocks [units_local, ...] into [num_units, ...]."""
    shape = local.shape[1:]
    pad = torch.zeros((plan.max_units,) + tuple(shape), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(plan.world)]
    dist.all_gather(bufs, pad.contiguous(), group=group)
    parts = []
    for r in range(plan.world):
        u0, u1 = plan.unit_range(r)
        parts.append(bufs[r][: u1 - u0])
    return torch.cat(parts, 0)


def _plan_for(q, k, group):
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    return ShardPlan(q.shape[0], q.shape[1], k.shape[1], world, rank)


def sharded_forward(q, k, v, causal=False, slide_size=0, softmax_scale=None, group=None, fwd_fn=None):
    """Forward over this rank's units, then all-gather O and LSE on every rank.

    q, k, v are the full (replicated) tensors. Returns full (O, LSE).
    """
    fwd_fn = fwd_fn or _default_fwd
    plan = _plan_for(q, k, group)
    B, Hq, N, D = q.shape
    G = plan.group
    o_parts, l_parts = [], []
    for b, kv0, kv1 in plan.runs():
        qs = q[b : b + 1, kv0 * G : kv1 * G]
        o, lse = fwd_fn(qs, k[b : b + 1, kv0:kv1], v[b : b + 1, kv0:kv1], causal, slide_size, softmax_scale)
        o_parts.append(o.reshape(kv1 - kv0, G, N, D))
        l_parts.append(lse.reshape(kv1 - kv0, G, N))
    empty = (0, G, N)
    o_loc = torch.cat(o_parts, 0) if o_parts else q.new_empty(empty + (D,))
    l_loc = torch.cat(l_parts, 0) if l_parts else q.new_empty(empty, dtype=torch.float32)
    if plan.world == 1:
        o_all, l_all = o_loc, l_loc
    else:
        o_all = _gather_units(plan, o_loc, group)
        l_all = _gather_units(plan, l_loc, group)
    # unit u = b * H_KV + kv owns query heads [kv*G, (kv+1)*G) of batch b
    return o_all.reshape(B, Hq, N, D), l_all.reshape(B, Hq, N)


def sharded_backward(q, k, v, o, lse, do, causal=False, slide_size=0, softmax_scale=None, group=None,
                     bwd_fn=None):
    """Backward over this rank's units, then all-gather dQ, dK, dV on every rank."""
    bwd_fn = bwd_fn or _default_bwd
    plan = _plan_for(q, k, group)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    G = plan.group
    dq_p, dk_p, dv_p = [], [], []
    for b, kv0, kv1 in plan.runs():
        hs = slice(kv0 * G, kv1 * G)
        dq, dk, dv = bwd_fn(q[b : b + 1, hs], k[b : b + 1, kv0:kv1], v[b : b + 1, kv0:kv1],
                            o[b : b + 1, hs], lse[b : b + 1, hs], do[b : b + 1, hs],
                            causal, slide_size, softmax_scale)
        dq_p.append(dq.reshape(kv1 - kv0, G, N, D))
        dk_p.append(dk.reshape(kv1 - kv0, N, D))
        dv_p.append(dv.reshape(kv1 - kv0, N, D))
    dq_loc = torch.cat(dq_p, 0) if dq_p else q.new_empty((0, G, N, D))
    dk_loc = torch.cat(dk_p, 0) if dk_p else k.new_empty((0, N, D))
    dv_loc = torch.cat(dv_p, 0) if dv_p else v.new_empty((0, N, D))
    if plan.world > 1:
        dq_loc = _gather_units(plan, dq_loc, group)
        dk_loc = _gather_units(plan, dk_loc, group)
        dv_loc = _gather_units(plan, dv_loc, group)
    return (dq_loc.reshape(B, Hq, N, D), dk_loc.reshape(B, Hkv, N, D), dv_loc.reshape(B, Hkv, N, D))
