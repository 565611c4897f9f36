"""Multi-rank sharding over (batch, KV-head group) units, run as gloo ranks on
CPU. The per-unit compute is the numpy oracle standing in for the kernel (test
only): what is under test is the partitioning and the all-gather reassembly."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemma_triton_flash_attn.sharding import ShardPlan, sharded_backward, sharded_forward
from oracle.attention_oracle import attention_bwd, attention_fwd


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_fwd(q, k, v, causal, slide, scale):
    o, lse = attention_fwd(q.numpy(), k.numpy(), v.numpy(), causal, slide, scale)
    return torch.from_numpy(o), torch.from_numpy(lse)


def oracle_bwd(q, k, v, o, lse, do, causal, slide, scale):
    dq, dk, dv, _ = attention_bwd(q.numpy(), k.numpy(), v.numpy(), o.numpy(), lse.numpy(), do.numpy(),
                                  causal, slide, scale)
    return torch.from_numpy(dq), torch.from_numpy(dk), torch.from_numpy(dv)


@pytest.mark.parametrize("B,Hkv,world", [(1, 4, 2), (4, 2, 8), (3, 5, 4), (1, 1, 3), (2, 3, 2)])
def test_plan_covers_every_unit_once(B, Hkv, world):
    seen = []
    sizes = []
    for r in range(world):
        plan = ShardPlan(B, Hkv * 2, Hkv, world, r)
        u0, u1 = plan.unit_range()
        sizes.append(u1 - u0)
        for b, kv0, kv1 in plan.runs():
            seen += [b * Hkv + kv for kv in range(kv0, kv1)]
    assert seen == list(range(B * Hkv))
    assert max(sizes) - min(sizes) <= 1


def _inputs():
    g = torch.Generator().manual_seed(7)
    B, Hq, Hkv, N, D = 2, 6, 3, 33, 16
    q = torch.randn(B, Hq, N, D, generator=g)
    k = torch.randn(B, Hkv, N, D, generator=g)
    v = torch.randn(B, Hkv, N, D, generator=g)
    do = torch.randn(B, Hq, N, D, generator=g)
    return q, k, v, do


def _worker(rank, world, port, out_dir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, do = _inputs()
        o, lse = sharded_forward(q, k, v, True, 5, None, fwd_fn=oracle_fwd)
        dq, dk, dv = sharded_backward(q, k, v, o, lse, do, True, 5, None, bwd_fn=oracle_bwd)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), o=o.numpy(), lse=lse.numpy(), dq=dq.numpy(),
                 dk=dk.numpy(), dv=dv.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_matches_single_rank(tmp_path, world):
    port = _free_port()
    mp.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    q, k, v, do = _inputs()
    o, lse = oracle_fwd(q, k, v, True, 5, None)
    dq, dk, dv = oracle_bwd(q, k, v, o, lse, do, True, 5, None)
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"r{r}.npz"))
        for name, ref in (("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
            np.testing.assert_allclose(z[name], ref.numpy(), rtol=1e-5, atol=1e-5, err_msg=f"rank {r} {name}")


def _failing_worker(rank, world, port, out_dir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    q, k, v, do = _inputs()
    if rank == 1:
        # This rank fails on the host before its collective; it never joins.
        os._exit(3)
    try:
        sharded_forward(q, k, v, True, 5, None, fwd_fn=oracle_fwd)
        open(os.path.join(out_dir, "completed"), "w").close()
    except Exception as e:  # gloo reports the missing peer instead of hanging
        open(os.path.join(out_dir, "error"), "w").write(type(e).__name__)


def test_rank_failure_surfaces_as_error_not_hang(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    assert os.path.exists(os.path.join(tmp_path, "error"))
    assert not os.path.exists(os.path.join(tmp_path, "completed"))


@pytest.mark.parametrize("n,parts,causal,window", [(16384, 2, True, 0), (16384, 4, True, 1024), (1000, 3, True, 0),
                                                   (200, 2, True, 0), (4096, 2, False, 0)])
@pytest.mark.parametrize("kind", ["q", "k"])
def test_sequence_split_ranges_cover_and_balance(n, parts, causal, window, kind):
    from gemma_triton_flash_attn.sharding import balanced_row_ranges, tile_work

    r = balanced_row_ranges(n, parts, kind, causal, window)
    assert r[0][0] == 0 and r[-1][1] == n and len(r) == parts
    for (a0, a1), (b0, b1) in zip(r[:-1], r[1:]):
        assert a1 == b0 and a0 % 128 == 0 and a0 < a1
    w = tile_work(n, kind, causal, window)
    per = [sum(w[a // 128:(b + 127) // 128]) for a, b in r]
    if n >= 4096:
        assert max(per) <= 1.1 * min(per), per


def test_sequence_split_plan_assignment():
    from gemma_triton_flash_attn.sharding import SequenceSplitPlan

    plan = SequenceSplitPlan(1, 32, 4, 16384, 8, True, 0)
    a = [plan.assignment(r) for r in range(8)]
    assert [(x[0], x[1]) for x in a] == [(0, kv) for kv in range(4) for _ in range(2)]
    assert a[0][2] == a[2][2] and a[0][2] != a[1][2]
    with pytest.raises(ValueError):
        SequenceSplitPlan(1, 32, 4, 16384, 6, True, 0).split


def test_head_split_assignment():
    from gemma_triton_flash_attn.sharding import head_split_assignment

    got = [head_split_assignment(1, 32, 4, 8, r) for r in range(8)]
    assert got == [(0, kv, kv * 8 + p * 4, 4) for kv in range(4) for p in range(2)]
    with pytest.raises(ValueError):
        head_split_assignment(1, 12, 4, 8, 0)  # 3 heads per group, 2 ranks per unit


# ---------------------------------------------------------------- persistent-buffer unit sharding
def _unit_worker(rank, world, port, out_dir):
    from gemma_triton_flash_attn.sharding import UnitShardedAttention

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, do = _inputs()
        B, Hq, N, D = q.shape
        calls = []

        def fwd_fn(qs, ks, vs, o, lse):
            calls.append(("fwd", qs.shape[1]))
            oo, ll = oracle_fwd(qs, ks, vs, True, 5, None)
            o.copy_(oo)
            lse.copy_(ll)

        def bwd_fn(stage, qs, ks, vs, o, lse, dos, dq, dk, dv, delta, ws):
            # the stand-in reads only this rank's own O / LSE rows, as the kernels do
            calls.append((f"bwd{stage}", qs.shape[1]))
            gq, gk, gv = oracle_bwd(qs, ks, vs, o.clone(), lse.clone(), dos, True, 5, None)
            if stage == 0:
                dq.copy_(gq)
                delta.copy_((dos * o).sum(-1))
            else:
                dk.copy_(gk)
                dv.copy_(gv)

        att = UnitShardedAttention(B, Hq, k.shape[1], N, D, q.dtype, q.device, causal=True, slide_size=5,
                                   fwd_fn=fwd_fn, bwd_fn=bwd_fn)
        o, lse, dq, dk, dv = att.step(q, k, v, do)
        # a second step reuses the buffers
        o, lse, dq, dk, dv = att.step(q, k, v, do)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), o=o.numpy(), lse=lse.numpy(), dq=dq.numpy(),
                 dk=dk.numpy(), dv=dv.numpy(), runs=np.array(att.runs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 6])
def test_unit_sharded_attention_matches_single_rank(tmp_path, world):
    port = _free_port()
    mp.spawn(_unit_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    q, k, v, do = _inputs()
    o, lse = oracle_fwd(q, k, v, True, 5, None)
    dq, dk, dv = oracle_bwd(q, k, v, o, lse, do, True, 5, None)
    units = []
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"r{r}.npz"))
        units += [int(b) * 3 + kv for b, kv0, kv1 in z["runs"] for kv in range(kv0, kv1)]
        for name, ref in (("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
            np.testing.assert_allclose(z[name], ref.numpy(), rtol=1e-5, atol=1e-5, err_msg=f"rank {r} {name}")
    assert units == list(range(6))  # every (b, kv) unit computed by exactly one rank


def test_unit_sharded_attention_single_rank_runs():
    from gemma_triton_flash_attn.sharding import ShardPlan, UnitShardedAttention

    assert ShardPlan(2, 6, 3, 4, 0).num_units % 4 != 0
    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        # one rank owns all six units: one run per batch element
        att = UnitShardedAttention(2, 6, 3, 33, 16, torch.float32, "cpu", fwd_fn=lambda *a: None,
                                   bwd_fn=lambda *a: None)
        assert att.runs == [(0, 0, 3), (1, 0, 3)]
    finally:
        dist.destroy_process_group()


def _head_split_worker(rank, world, port, out_dir):
    from gemma_triton_flash_attn.sharding import UnitShardedAttention

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(9)
        q, k, v, do = (torch.randn(s, generator=g) for s in ((1, 8, 33, 16), (1, 2, 33, 16), (1, 2, 33, 16),
                                                             (1, 8, 33, 16)))

        def fwd_fn(qs, ks, vs, o, lse):
            oo, ll = oracle_fwd(qs, ks, vs, True, 0, None)
            o.copy_(oo)
            lse.copy_(ll)

        def partial_fn(qs, ks, vs, o, lse, dos, dq, dk32, dv32, delta, ws):
            gq, gk, gv = oracle_bwd(qs, ks, vs, o.clone(), lse.clone(), dos, True, 0, None)
            dq.copy_(gq)
            dk32.copy_(gk)  # this rank's heads' share of the KV head's gradient
            dv32.copy_(gv)

        att = UnitShardedAttention(1, 8, 2, 33, 16, torch.float32, "cpu", causal=True, fwd_fn=fwd_fn,
                                   partial_fn=partial_fn)
        assert att.split == world // 2
        for _ in range(2):
            o, lse, dq, dk, dv = att.step(q, k, v, do)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), o=o.numpy(), lse=lse.numpy(), dq=dq.numpy(),
                 dk=dk.numpy(), dv=dv.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [4, 8])
def test_unit_sharded_attention_head_split_matches_single_rank(tmp_path, world):
    """More ranks than (batch, KV-head) units: each unit's query heads split
    over world / units ranks, the dK/dV partials summed within the unit's ranks."""
    port = _free_port()
    mp.spawn(_head_split_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    g = torch.Generator().manual_seed(9)
    q, k, v, do = (torch.randn(s, generator=g) for s in ((1, 8, 33, 16), (1, 2, 33, 16), (1, 2, 33, 16),
                                                         (1, 8, 33, 16)))
    o, lse = oracle_fwd(q, k, v, True, 0, None)
    dq, dk, dv = oracle_bwd(q, k, v, o, lse, do, True, 0, None)
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"r{r}.npz"))
        for name, ref in (("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
            np.testing.assert_allclose(z[name], ref.numpy(), rtol=1e-5, atol=1e-5, err_msg=f"rank {r} {name}")
