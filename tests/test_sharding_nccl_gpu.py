"""(batch, KV-group) sharding over NCCL on 2+ GPUs: each rank computes its
units with the kernels and all-gathers the outputs; every rank must hold the
single-GPU result. Skipped when fewer than two GPUs are visible."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import assert_close, torch_ref

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(device, split=False):
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, N, D = (1, 8, 1, 1000, 512) if split else (2, 16, 2, 640, 512)
    mk = lambda *s: (torch.randn(*s, generator=g) * 0.5).bfloat16().to(device)  # noqa: E731
    return mk(B, Hq, N, D), mk(B, Hkv, N, D), mk(B, Hkv, N, D), mk(B, Hq, N, D)


def _worker(rank, world, port, out_dir, split=False):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        from gemma_triton_flash_attn import sharding as sh

        q, k, v, do = _inputs(f"cuda:{rank}", split in ("seq", "heads", "persistent_heads"))
        if split in ("persistent", "persistent_ce", "persistent_heads"):
            att = sh.UnitShardedAttention(q.shape[0], q.shape[1], k.shape[1], q.shape[2], q.shape[3], q.dtype,
                                          q.device, causal=True, gather="ce" if split == "persistent_ce" else "nccl")
            for _ in range(2):  # the second step reuses every buffer
                o, lse, dq, dk, dv = att.step(q, k, v, do)
            torch.cuda.synchronize()
            torch.save({n: t.cpu() for n, t in dict(o=o, lse=lse, dq=dq, dk=dk, dv=dv).items()},
                       os.path.join(out_dir, f"r{rank}.pt"))
            return
        fwd, bwd = {False: (sh.sharded_forward, sh.sharded_backward), "seq": (sh.split_forward, sh.split_backward),
                    "heads": (sh.head_split_forward, sh.head_split_backward)}[split]
        o, lse = fwd(q, k, v, True, 0)
        dq, dk, dv = bwd(q, k, v, o, lse, do, True, 0)
        torch.save({n: t.cpu() for n, t in dict(o=o, lse=lse, dq=dq, dk=dk, dv=dv).items()},
                   os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", [False, "persistent", "persistent_ce", "seq", "heads", "persistent_heads"],
                         ids=["units", "unit_sharded_attention", "unit_sharded_attention_copy_engines",
                              "sequence_split", "head_split", "unit_sharded_attention_head_split"])
def test_sharded_equals_single_gpu(tmp_path, split, monkeypatch):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    if split in ("seq", "heads", "persistent_heads"):
        world = 2  # one (batch, KV-group) unit split over two ranks by sequence blocks
    from gemma_triton_flash_attn.attention import flash_attn_gqa_backward, flash_attn_gqa_forward_with_lse

    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), split), nprocs=world, join=True)
    q, k, v, do = _inputs("cuda:0", split in ("seq", "heads", "persistent_heads"))
    o, lse = flash_attn_gqa_forward_with_lse(q, k, v, True, 0)
    if split == "seq":
        # the sequence split runs the recomputing kernels (row-range entries):
        # compare with the same kernels on one GPU
        monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "0")
    dq, dk, dv = flash_attn_gqa_backward(q, k, v, o, lse, do, True, 0)
    ref = dict(o=o, lse=lse, dq=dq, dk=dk, dv=dv)
    if split in ("heads", "persistent_heads"):
        r32 = torch_ref(q, k, v, do, True, 0)
        m32 = torch_ref(q, k, v, do, True, 0, magnitudes=True)
        ref32 = dict(zip(("o", "lse", "dq", "dk", "dv"), r32))
        mag32 = dict(zip(("o", "lse", "dq", "dk", "dv"), m32))
    for r in range(world):
        got = torch.load(os.path.join(tmp_path, f"r{r}.pt"))
        for n, t in ref.items():
            if split in ("heads", "persistent_heads") and n in ("dk", "dv"):
                # The sum of the ranks' fp32 partials (another summation order than
                # one GPU's, rounded once) is held to the suite's criterion
                # against fp32.
                assert_close(f"rank {r} {n}", got[n], ref32[n], magnitude=mag32[n])
            else:
                d = (got[n].float() - t.float().cpu()).abs().max().item()
                assert torch.equal(got[n], t.cpu()), f"rank {r} {n}: max diff {d:.3e}"  # same kernels: bitwise
