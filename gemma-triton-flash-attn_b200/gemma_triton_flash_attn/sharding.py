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

import functools
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["ShardPlan", "sharded_forward", "sharded_backward", "UnitShardedAttention", "SequenceSplitPlan",
           "balanced_row_ranges", "split_forward", "split_backward", "head_split_assignment", "head_split_forward",
           "head_split_backward"]


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


# --------------------------------------------------------------------------
# Persistent-buffer unit sharding with overlapped all-gathers
# --------------------------------------------------------------------------


class UnitShardedAttention:
    """Forward + backward of one attention problem over the ranks of `group`,
    each rank computing whole (batch, KV-head) units, with the outputs
    reassembled on every rank by all-gathers that run while the next kernels
    compute.

    The output tensors (O, LSE, dQ, dK, dV, delta) are allocated once, full
    size and contiguous. Units are numbered u = b * H_KV + kv_head, so the
    query heads of a block of consecutive units are one contiguous range of the
    flattened (B * H_Q, N, D) storage: every rank's kernels write straight
    into its own slice and an in-place ``all_gather_into_tensor`` fills the
    other ranks' slices. No copies are made on either side.

    Order of work on the calling stream, with the collectives on the process
    group's own stream:

        forward kernels -> all-gather O, LSE      (overlaps the backward kernels)
        dQ + P/dS kernels -> all-gather dQ        (overlaps the dK/dV kernels)
        dK/dV kernels -> all-gather dK, dV
        ``wait()``: the calling stream waits for the four collectives

    Needs B * H_KV to be a multiple of the world size (equal blocks, which the
    in-place all-gather needs), or the world size a multiple of B * H_KV with
    the G query heads of a unit divisible by s = world / (B * H_KV): then
    ("head split") the s ranks of a unit each take G/s of its query heads
    (their heads are still one rank-ordered slice of the flattened storage,
    so O, LSE and dQ are gathered the same way), each writes its dK/dV share
    as an fp32 partial (``gqafa_bwd_partial``), the s partials are summed by
    an all-reduce within the unit's ranks, rounded once and all-gathered.
    ``sharded_forward`` / ``sharded_backward`` handle uneven splits. The per-unit kernels are the materialised backward
    (``gqafa_bwd_ws``) with one workspace per contiguous run of units, so the
    dQ stage of every run can precede all dK/dV stages.

    ``fwd_fn(q, k, v, o, lse)`` and ``bwd_fn(stage, q, k, v, o, lse, do, dq,
    dk, dv, delta, workspace)`` replace the kernels (CPU tests); by default
    they are this library's CUDA launches.

    ``gather="ce"`` (GPUs only) replaces the NCCL all-gathers by copy-engine
    pushes over NVLink: the output buffers are symmetric memory
    (torch.distributed._symmetric_memory), every rank copies its own slice
    into the same slice of every peer's buffer with cudaMemcpyAsync on its own
    copy streams, and ``wait()`` ends with a one-element NCCL all-reduce that
    orders every rank after all pushes. Copy engines use no SMs, so the
    gathers take nothing from the kernels they overlap. A step's outputs stay
    valid until the next ``step`` / ``forward`` on any rank (peers push into
    them).
    """

    def __init__(self, batch, heads_q, heads_kv, seqlen, head_dim, dtype, device, causal=True, slide_size=0,
                 softmax_scale=None, group=None, fwd_fn=None, bwd_fn=None, gather="nccl", copy_streams=4,
                 partial_fn=None):
        from .attention import _normalize_window

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.plan = ShardPlan(batch, heads_q, heads_kv, self.world, self.rank)
        units, G = self.plan.num_units, heads_q // heads_kv
        self.split = 1  # ranks per unit (head split when > 1)
        if units % self.world != 0:
            s = self.world // units
            if self.world % units != 0 or G % s != 0:
                raise ValueError(f"{units} (batch, KV-head) units with {G} query heads each do not divide over "
                                 f"{self.world} ranks")
            self.split = s
        self.shape = (batch, heads_q, heads_kv, seqlen, head_dim)
        self.causal = bool(causal)
        self.window = _normalize_window(causal, slide_size, seqlen)
        self.scale = (1.0 / math.sqrt(head_dim)) if softmax_scale is None else float(softmax_scale)
        B, Hq, Hkv, N, D = self.shape
        if gather not in ("nccl", "ce"):
            raise ValueError(f"gather must be 'nccl' or 'ce', got {gather!r}")
        self.gather = gather if self.world > 1 else "nccl"
        alloc = torch.empty
        if self.gather == "ce":
            import torch.distributed._symmetric_memory as symm

            alloc = lambda shape, dtype, device: symm.empty(shape, dtype=dtype, device=device)  # noqa: E731
        self.o = alloc((B, Hq, N, D), dtype=dtype, device=device)
        self.dq = alloc((B, Hq, N, D), dtype=dtype, device=device)
        self.dk = alloc((B, Hkv, N, D), dtype=dtype, device=device)
        self.dv = alloc((B, Hkv, N, D), dtype=dtype, device=device)
        self.lse = alloc((B, Hq, N), dtype=torch.float32, device=device)
        self.delta = torch.empty((B, Hq, N), dtype=torch.float32, device=device)
        self._peers = {}
        if self.gather == "ce":
            pg = group if group is not None else dist.group.WORLD
            for name in ("o", "dq", "dk", "dv", "lse"):
                t = getattr(self, name)
                hdl = symm.rendezvous(t, pg)
                self._peers[name] = [hdl.get_buffer(p, tuple(t.shape), t.dtype) for p in range(self.world)]
            self._copy_streams = [torch.cuda.Stream(device) for _ in range(copy_streams)]
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        if self.split == 1:
            self.runs = list(self.plan.runs())
        else:
            unit, part = divmod(self.rank, self.split)
            b, kv = divmod(unit, Hkv)
            self.runs = [(b, kv, kv + 1)]
            self._heads = (kv * G + part * (G // self.split), G // self.split)
            self._unit = unit
            self._dkv32 = torch.empty((2, 1, 1, N, D), dtype=torch.float32, device=device)
            self._dkv_all = torch.empty((self.world, 2, N, D), dtype=dtype, device=device)
            self._subgroup = _unit_subgroup(group, units, self.split, unit) if self.world > 1 else None
        self._fwd_fn = fwd_fn or self._kernel_fwd
        self._bwd_fn = bwd_fn or self._kernel_bwd
        self._partial_fn = partial_fn or self._kernel_partial
        self.workspaces = None
        if self.split > 1 and partial_fn is None:
            from .attention import _alloc_workspace, bwd_workspace_size

            nh = self._heads[1]
            self.workspaces = [_alloc_workspace(bwd_workspace_size(1, nh, 1, N, D, self.causal, self.window), device)]
        elif self.split == 1 and bwd_fn is None:
            from .attention import _alloc_workspace, bwd_workspace_size

            G = Hq // Hkv
            self.workspaces = []
            for _, kv0, kv1 in self.runs:
                size = bwd_workspace_size(1, (kv1 - kv0) * G, kv1 - kv0, N, D, self.causal, self.window)
                ws = _alloc_workspace(size, device)
                if ws is None and size > 0:
                    raise MemoryError(f"no room for the {size}-byte backward workspace of a run of units")
                self.workspaces.append(ws)
        self._works = []

    # ---- kernels -------------------------------------------------------------
    def _kernel_fwd(self, q, k, v, o, lse):
        from .attention import _fwd

        _fwd(q, k, v, self.causal, self.window, self.scale, True, out=(o, lse))

    def _kernel_bwd(self, stage, q, k, v, o, lse, do, dq, dk, dv, delta, workspace):
        from .attention import _bwd

        _bwd(q, k, v, o, lse, do, self.causal, self.window, self.scale, stage=stage, out=(dq, dk, dv, delta),
             workspace=workspace)

    def _kernel_partial(self, q, k, v, o, lse, do, dq, dk32, dv32, delta, workspace):
        from . import _lib
        from .attention import _bwd_args

        tail = (workspace.data_ptr(), workspace.numel()) if workspace is not None else (None, 0)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.load().gqafa_bwd_partial(
            *_bwd_args(q, k, v, o, do, lse, dq, dk32, dv32, delta, self.causal, self.window, self.scale, stream),
            *tail))

    # ---- slices --------------------------------------------------------------
    def _qv(self, i, t):
        """Run i's query heads of a [B, H_Q, ...] tensor (a view)."""
        b, kv0, kv1 = self.runs[i]
        if self.split > 1:
            h0, nh = self._heads
            return t[b:b + 1, h0:h0 + nh]
        G = self.plan.group
        return t[b:b + 1, kv0 * G:kv1 * G]

    def _kvv(self, i, t):
        """Run i's KV heads of a [B, H_KV, ...] tensor (a view)."""
        b, kv0, kv1 = self.runs[i]
        return t[b:b + 1, kv0:kv1]

    def _gather(self, t, name=None):
        """Start the all-gather of this rank's block of `t` (flattened over
        batch and heads, which are unit-ordered): in place with NCCL, or as
        copy-engine pushes into the peers' symmetric buffers."""
        if self.world == 1:
            return
        flat = t.view(self.world, -1)
        if self.gather == "nccl":
            self._works.append(dist.all_gather_into_tensor(t.view(-1), flat[self.rank], group=self.group,
                                                           async_op=True))
            return
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(t.device))
        mine = flat[self.rank]
        ns = len(self._copy_streams)
        for j in range(1, self.world):  # peers in rotated order, spread over the copy streams
            p = (self.rank + j) % self.world
            s = self._copy_streams[(j - 1) % ns]
            s.wait_event(ready)
            with torch.cuda.stream(s):
                self._peers[name][p].view(self.world, -1)[self.rank].copy_(mine, non_blocking=True)

    # ---- passes --------------------------------------------------------------
    def forward(self, q, k, v):
        """O and LSE of this rank's units, then their all-gather (started, not awaited)."""
        for i in range(len(self.runs)):
            self._fwd_fn(self._qv(i, q), self._kvv(i, k), self._kvv(i, v), self._qv(i, self.o), self._qv(i, self.lse))
        self._gather(self.o, "o")
        self._gather(self.lse, "lse")
        return self.o, self.lse

    def backward(self, q, k, v, do):
        """dQ, dK, dV of this rank's units (from this rank's own O / LSE rows,
        which the all-gather does not touch), each followed by its all-gather."""
        if self.split > 1:
            return self._backward_head_split(q, k, v, do)
        n = len(self.runs)
        for stage in (0, 1):
            for i in range(n):
                qv, kvv = (lambda t: self._qv(i, t)), (lambda t: self._kvv(i, t))
                ws = self.workspaces[i] if self.workspaces is not None else None
                self._bwd_fn(stage, qv(q), kvv(k), kvv(v), qv(self.o), qv(self.lse), qv(do), qv(self.dq),
                             kvv(self.dk), kvv(self.dv), qv(self.delta), ws)
            if stage == 0:
                self._gather(self.dq, "dq")
        self._gather(self.dk, "dk")
        self._gather(self.dv, "dv")
        return self.dq, self.dk, self.dv

    def _backward_head_split(self, q, k, v, do):
        qv, kvv = (lambda t: self._qv(0, t)), (lambda t: self._kvv(0, t))
        ws = self.workspaces[0] if self.workspaces is not None else None
        self._partial_fn(qv(q), kvv(k), kvv(v), qv(self.o), qv(self.lse), qv(do), qv(self.dq), self._dkv32[0],
                         self._dkv32[1], qv(self.delta), ws)
        self._gather(self.dq, "dq")
        if self.world > 1:
            dist.all_reduce(self._dkv32, group=self._subgroup)  # the unit's s partials
            mine = self._dkv32.view(2, *self._dkv32.shape[-2:]).to(self._dkv_all.dtype)
            out = self._dkv_all.view(-1, *self._dkv_all.shape[-2:])  # (world * 2, N, D): chunks along dim 0
            self._works.append(dist.all_gather_into_tensor(out, mine, group=self.group, async_op=True))
        else:
            self._dkv_all[0].copy_(self._dkv32.view(self._dkv_all.shape[1:]))
        return self.dq, self.dk, self.dv

    def wait(self):
        """Make the calling stream wait for every collective started so far."""
        if self.gather == "ce" and self.world > 1:
            cur = torch.cuda.current_stream(self._flag.device)
            for s in self._copy_streams:
                cur.wait_stream(s)
            # every rank's pushes are complete once every rank has reached this
            # all-reduce (each enqueues it after its own copies)
            self._works.append(dist.all_reduce(self._flag, group=self.group, async_op=True))
        for w in self._works:
            w.wait()
        self._works = []
        if self.split > 1:  # one copy of each unit's summed dK, dV
            Hkv = self.shape[2]
            for u in range(self.plan.num_units):
                ub, ukv = divmod(u, Hkv)
                self.dk[ub, ukv].copy_(self._dkv_all[u * self.split, 0])
                self.dv[ub, ukv].copy_(self._dkv_all[u * self.split, 1])

    def step(self, q, k, v, do):
        """One full forward + backward with every output reassembled on every rank."""
        self.forward(q, k, v)
        self.backward(q, k, v, do)
        self.wait()
        return self.o, self.lse, self.dq, self.dk, self.dv


# --------------------------------------------------------------------------
# Sequence split: more ranks than (batch, KV-group) units
# --------------------------------------------------------------------------
#
# Config 2 at 8 GPUs has only B * H_KV = 4 units. Each unit is then split over
# s = world / units ranks by blocks of 128 rows: a rank computes the O / LSE
# and dQ rows of its query range, and the dK / dV rows of its key range. The
# key-range stages read LSE and delta of every query row of the unit, so LSE
# (after the forward) and delta (after the dQ stage) are all-gathered in
# between; they are B * H_Q * N floats, small next to the outputs. Ranges are
# chosen so that every rank of a unit gets about the same causal work.

TILE = 128


def tile_work(n: int, kind: str, causal: bool, window: int) -> list[int]:
    """Attended pairs per 128-row tile: of its query rows (kind "q") or of its key rows (kind "k")."""
    out = []
    for t0 in range(0, n, TILE):
        w = 0
        for r in range(t0, min(n, t0 + TILE)):
            if not causal:
                w += n
            elif kind == "q":
                w += min(r + 1, window) if window else r + 1
            else:
                w += (min(n, r + window) if window else n) - r
        out.append(w)
    return out


@functools.lru_cache(maxsize=256)
def balanced_row_ranges(n: int, parts: int, kind: str, causal: bool, window: int) -> list[tuple[int, int]]:
    """Split [0, n) into `parts` contiguous ranges on 128-row boundaries with
    about equal attention work; every range is non-empty when possible."""
    work = tile_work(n, kind, causal, window)
    tiles = len(work)
    if parts > tiles:
        raise ValueError(f"cannot split {tiles} row tiles into {parts} parts")
    total = float(sum(work))
    bounds, acc, t = [0], 0.0, 0
    for part in range(1, parts):
        target = total * part / parts
        # advance while the next tile keeps us at or below the target, leaving
        # at least one tile for each remaining part
        while t < tiles - (parts - part) and acc + work[t] / 2 <= target:
            acc += work[t]
            t += 1
        t = max(t, bounds[-1] + 1)
        bounds.append(t)
    bounds.append(tiles)
    return [(b0 * TILE, min(n, b1 * TILE)) for b0, b1 in zip(bounds[:-1], bounds[1:])]


@dataclass(frozen=True)
class SequenceSplitPlan:
    batch: int
    heads_q: int
    heads_kv: int
    seqlen: int
    world: int
    causal: bool
    window: int

    @property
    def units(self) -> int:
        return self.batch * self.heads_kv

    @property
    def split(self) -> int:
        if self.world % self.units != 0 or self.world < self.units:
            raise ValueError(f"world {self.world} must be a multiple of the {self.units} (batch, KV-group) units")
        return self.world // self.units

    @functools.lru_cache(maxsize=1024)  # noqa: B019 - plans are small, frozen and few
    def assignment(self, rank: int):
        """(b, kv_head, query rows, key rows) of `rank`."""
        s = self.split
        unit, part = divmod(rank, s)
        b, kv = divmod(unit, self.heads_kv)
        q_rows = balanced_row_ranges(self.seqlen, s, "q", self.causal, self.window)[part]
        k_rows = balanced_row_ranges(self.seqlen, s, "k", self.causal, self.window)[part]
        return b, kv, q_rows, k_rows


def _gather_rows(plan, local: torch.Tensor, row_dim: int, which: str, group=None):
    """All-gather each rank's row block (rows along `row_dim`) into a list
    indexed by rank, each trimmed to that rank's row count."""
    world = plan.world
    idx = 2 if which == "q" else 3
    counts = [plan.assignment(r)[idx][1] - plan.assignment(r)[idx][0] for r in range(world)]
    m = max(counts)
    shape = list(local.shape)
    shape[row_dim] = m
    pad = torch.zeros(shape, dtype=local.dtype, device=local.device)
    pad.narrow(row_dim, 0, local.shape[row_dim]).copy_(local)
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return [bufs[r].narrow(row_dim, 0, counts[r]) for r in range(world)]


def split_forward(q, k, v, causal=False, slide_size=0, softmax_scale=None, group=None):
    """Forward with each (batch, KV-group) unit split over several ranks by
    query rows; returns the full (O, LSE) on every rank."""
    from .attention import _check_inputs, _fwd, _normalize_window

    _check_inputs(q, k, v)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    window = _normalize_window(causal, slide_size, N)
    scale = (1.0 / math.sqrt(D)) if softmax_scale is None else float(softmax_scale)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    plan = SequenceSplitPlan(B, Hq, Hkv, N, world, bool(causal), window)
    b, kv, (q0, q1), _ = plan.assignment(rank)
    hs = slice(kv * G, (kv + 1) * G)
    qs, ks, vs = q[b:b + 1, hs], k[b:b + 1, kv:kv + 1], v[b:b + 1, kv:kv + 1]
    o_loc = torch.empty_like(qs).contiguous()
    lse_loc = torch.empty((1, G, N), dtype=torch.float32, device=q.device)
    _fwd(qs, ks, vs, causal, window, scale, True, rows=(q0, q1), out=(o_loc, lse_loc))
    o_parts = _gather_rows(plan, o_loc[:, :, q0:q1].contiguous(), 2, "q", group)
    l_parts = _gather_rows(plan, lse_loc[:, :, q0:q1].contiguous(), 2, "q", group)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, N), dtype=torch.float32, device=q.device)
    for r in range(world):
        rb, rkv, (r0, r1), _ = plan.assignment(r)
        o[rb:rb + 1, rkv * G:(rkv + 1) * G, r0:r1] = o_parts[r]
        lse[rb:rb + 1, rkv * G:(rkv + 1) * G, r0:r1] = l_parts[r]
    return o, lse


def split_backward(q, k, v, o, lse, do, causal=False, slide_size=0, softmax_scale=None, group=None):
    """Backward of split_forward: dQ rows by query range, then (after
    all-gathering delta) dK / dV rows by key range; full gradients on every rank."""
    from .attention import _bwd, _check_inputs, _normalize_window

    _check_inputs(q, k, v)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    window = _normalize_window(causal, slide_size, N)
    scale = (1.0 / math.sqrt(D)) if softmax_scale is None else float(softmax_scale)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    plan = SequenceSplitPlan(B, Hq, Hkv, N, world, bool(causal), window)
    b, kv, (q0, q1), (k0, k1) = plan.assignment(rank)
    hs = slice(kv * G, (kv + 1) * G)
    args = (q[b:b + 1, hs], k[b:b + 1, kv:kv + 1], v[b:b + 1, kv:kv + 1], o[b:b + 1, hs],
            lse[b:b + 1, hs].contiguous(), do[b:b + 1, hs])
    dq_loc = torch.empty((1, G, N, D), dtype=q.dtype, device=q.device)
    dk_loc = torch.empty((1, 1, N, D), dtype=k.dtype, device=q.device)
    dv_loc = torch.empty((1, 1, N, D), dtype=v.dtype, device=q.device)
    delta = torch.empty((1, G, N), dtype=torch.float32, device=q.device)
    bufs = (dq_loc, dk_loc, dv_loc, delta)
    _bwd(*args, causal, window, scale, stage=0, out=bufs, rows=(q0, q1))
    d_parts = _gather_rows(plan, delta[:, :, q0:q1].contiguous(), 2, "q", group)
    for r in range(world):
        rb, rkv, (r0, r1), _ = plan.assignment(r)
        if (rb, rkv) == (b, kv):
            delta[:, :, r0:r1] = d_parts[r]
    _bwd(*args, causal, window, scale, stage=1, out=bufs, rows=(k0, k1))
    _bwd(*args, causal, window, scale, stage=2, out=bufs, rows=(k0, k1))
    dq_parts = _gather_rows(plan, dq_loc[:, :, q0:q1].contiguous(), 2, "q", group)
    dk_parts = _gather_rows(plan, dk_loc[:, :, k0:k1].contiguous(), 2, "k", group)
    dv_parts = _gather_rows(plan, dv_loc[:, :, k0:k1].contiguous(), 2, "k", group)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    for r in range(world):
        rb, rkv, (r0, r1), (s0, s1) = plan.assignment(r)
        dq[rb:rb + 1, rkv * G:(rkv + 1) * G, r0:r1] = dq_parts[r]
        dk[rb:rb + 1, rkv:rkv + 1, s0:s1] = dk_parts[r]
        dv[rb:rb + 1, rkv:rkv + 1, s0:s1] = dv_parts[r]
    return dq, dk, dv


# --------------------------------------------------------------------------
# Head split: more ranks than units, each unit's query heads divided
# --------------------------------------------------------------------------
#
# The preferred way to use more ranks than (batch, KV-group) units: the s
# ranks of a unit each take G/s of its query heads over the whole sequence.
# Forward and dQ need nothing from the other ranks; dK and dV of the unit's KV
# head are the sum of the s ranks' partial results (each over its G/s heads),
# the path's one real reduction: the kernels write the partials in fp32
# (gqafa_bwd_partial) and they are summed by an all-reduce within the unit's
# ranks before the one rounding to the input dtype. Every kernel
# keeps its full-sequence grid, unlike the sequence split, whose dK/dV launches
# shrink to one KV head and a fraction of its rows.


def head_split_assignment(batch: int, heads_q: int, heads_kv: int, world: int, rank: int):
    """(b, kv_head, first query head, number of query heads) of `rank`."""
    units = batch * heads_kv
    if world % units != 0 or world < units:
        raise ValueError(f"world {world} must be a multiple of the {units} (batch, KV-group) units")
    s = world // units
    g = heads_q // heads_kv
    if g % s != 0:
        raise ValueError(f"{s} ranks per unit do not divide its {g} query heads")
    unit, part = divmod(rank, s)
    b, kv = divmod(unit, heads_kv)
    return b, kv, kv * g + part * (g // s), g // s


def head_split_forward(q, k, v, causal=False, slide_size=0, softmax_scale=None, group=None):
    """Forward with each unit's query heads divided over s ranks; full (O, LSE) on every rank."""
    from .attention import flash_attn_gqa_forward_with_lse

    B, Hq, N, D = q.shape
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    b, kv, h0, nh = head_split_assignment(B, Hq, k.shape[1], world, rank)
    o_loc, l_loc = flash_attn_gqa_forward_with_lse(q[b:b + 1, h0:h0 + nh], k[b:b + 1, kv:kv + 1],
                                                   v[b:b + 1, kv:kv + 1], causal, slide_size, softmax_scale)
    o_parts = [torch.empty_like(o_loc) for _ in range(world)]
    l_parts = [torch.empty_like(l_loc) for _ in range(world)]
    dist.all_gather(o_parts, o_loc.contiguous(), group=group)
    dist.all_gather(l_parts, l_loc.contiguous(), group=group)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, N), dtype=torch.float32, device=q.device)
    for r in range(world):
        rb, _, rh0, rnh = head_split_assignment(B, Hq, k.shape[1], world, r)
        o[rb:rb + 1, rh0:rh0 + rnh] = o_parts[r]
        lse[rb:rb + 1, rh0:rh0 + rnh] = l_parts[r]
    return o, lse


_SUBGROUPS = {}


def _unit_subgroup(group, units, s, unit):
    """The process group of the s ranks of `unit` (created once, by every rank
    for every unit in the same order, as torch.distributed requires)."""
    granks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    key = (tuple(granks), s)
    if key not in _SUBGROUPS:
        _SUBGROUPS[key] = [dist.new_group([granks[u * s + j] for j in range(s)]) for u in range(units)]
    return _SUBGROUPS[key][unit]


def _partial_backward(q, k, v, o, lse, do, causal, window, scale):
    """dQ in the input dtype and dK, dV as fp32 partials (gqafa_bwd_partial:
    the materialised backward when its workspace fits, else the recomputing
    one), for a rank that holds some of the query heads of a KV group."""
    from . import _lib
    from .attention import _abi_ready, _alloc_workspace, _bwd_args, bwd_workspace_size

    b, h_q, n, d = q.shape
    h_kv = k.shape[1]
    q, k, v, o, do = (_abi_ready(t) for t in (q, k, v, o, do))
    dq = torch.empty_like(q)
    dk = torch.empty(k.shape, dtype=torch.float32, device=q.device)
    dv = torch.empty(v.shape, dtype=torch.float32, device=q.device)
    delta = torch.empty((b, h_q, n), dtype=torch.float32, device=q.device)
    ws = _alloc_workspace(bwd_workspace_size(b, h_q, h_kv, n, d, causal, window), q.device)
    tail = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _lib.check(_lib.load().gqafa_bwd_partial(
        *_bwd_args(q, k, v, o, do, lse.contiguous(), dq, dk, dv, delta, causal, window, scale, stream), *tail))
    return dq, dk, dv


def head_split_backward(q, k, v, o, lse, do, causal=False, slide_size=0, softmax_scale=None, group=None):
    """Backward of head_split_forward: dQ per rank; dK/dV of each unit are the
    sum of its s ranks' fp32 partials (an all-reduce within those s ranks
    only, before any rounding), then rounded once and all-gathered; full
    gradients on every rank."""
    from .attention import _check_inputs, _normalize_window

    _check_inputs(q, k, v)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    window = _normalize_window(causal, slide_size, N)
    scale = (1.0 / math.sqrt(D)) if softmax_scale is None else float(softmax_scale)
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    b, kv, h0, nh = head_split_assignment(B, Hq, Hkv, world, rank)
    units = B * Hkv
    s = world // units
    hs = slice(h0, h0 + nh)
    dq_loc, dk_p, dv_p = _partial_backward(
        q[b:b + 1, hs], k[b:b + 1, kv:kv + 1], v[b:b + 1, kv:kv + 1], o[b:b + 1, hs],
        lse[b:b + 1, hs], do[b:b + 1, hs], causal, window, scale)
    dq_parts = [torch.empty_like(dq_loc) for _ in range(world)]
    dist.all_gather(dq_parts, dq_loc.contiguous(), group=group)
    dq = torch.empty_like(q)
    for r in range(world):
        rb, _, rh0, rnh = head_split_assignment(B, Hq, Hkv, world, r)
        dq[rb:rb + 1, rh0:rh0 + rnh] = dq_parts[r]
    dkv = torch.stack((dk_p[0, 0], dv_p[0, 0]))  # (2, N, D) fp32 partial of this rank's heads
    if s > 1:
        dist.all_reduce(dkv, group=_unit_subgroup(group, units, s, rank // s))
    mine = dkv.to(k.dtype)
    gathered = torch.empty((world,) + tuple(mine.shape), dtype=k.dtype, device=q.device)
    dist.all_gather_into_tensor(gathered, mine, group=group)
    dk, dv = torch.empty_like(k), torch.empty_like(v)
    for u in range(units):
        ub, ukv = divmod(u, Hkv)
        dk[ub, ukv] = gathered[u * s, 0]
        dv[ub, ukv] = gathered[u * s, 1]
    return dq, dk, dv
