"""The materialised backward (head_dim 256 and 512) (gqafa_bwd_ws: the dQ kernel stores P
and dS, one kernel computes dK and dV from them) against the fp32 reference and
against the recomputing backward (gqafa_bwd), on causal, sliding-window,
non-causal, ragged and GQA shapes."""
import math

import pytest
import torch

from gemma_triton_flash_attn import _lib
from gemma_triton_flash_attn.attention import _bwd, _fwd, bwd_workspace_size
from helpers import assert_close, make_inputs, torch_ref

pytestmark = pytest.mark.gpu

DEV = "cuda"

CASES = [
    # (B, Hq, Hkv, N, causal, window, dtype)
    (1, 4, 1, 300, True, 0, torch.bfloat16),
    (2, 4, 2, 200, False, 0, torch.float16),
    (1, 2, 1, 1000, True, 300, torch.bfloat16),
    (1, 4, 2, 777, True, 129, torch.float16),
    (1, 8, 2, 2048, True, 0, torch.bfloat16),
    (1, 2, 2, 129, True, 0, torch.bfloat16),
    (1, 2, 1, 64, False, 0, torch.bfloat16),
]


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert _lib.device_status(torch.cuda.current_device(), reset=True) == 0, "a kernel wait timed out"


def _run(B, Hq, Hkv, N, causal, window, dt, seed=0, D=512):
    q, k, v, do = (t.to(DEV) for t in make_inputs(B, Hq, Hkv, N, D, dtype=dt, factor=0.5, seed=seed))
    scale = 1.0 / math.sqrt(D)
    o, lse = _fwd(q, k, v, causal, window, scale, True)
    size = bwd_workspace_size(B, Hq, Hkv, N, D, causal, window)
    assert size > 0
    # garbage in the workspace must not matter: every read block is written first
    ws = torch.full((size,), 0xFF, dtype=torch.uint8, device=DEV)
    got = _bwd(q, k, v, o, lse, do, causal, window, scale, workspace=ws)
    # the recomputing kernels one stage at a time; dK (stage 1) reads the
    # delta stage 0 wrote, so all stages share one buffer set
    bufs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty(B, Hq, N, device=DEV))
    for s in range(3):
        _bwd(q, k, v, o, lse, do, causal, window, scale, stage=s, out=bufs)
    rec = bufs[:3]
    torch.cuda.synchronize()
    return (q, k, v, do, scale), got, rec


@pytest.mark.parametrize("D", [256, 512])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}H{c[1]}x{c[2]}N{c[3]}c{int(c[4])}w{c[5]}")
def test_ws_matches_reference(case, D):
    B, Hq, Hkv, N, causal, window, dt = case
    (q, k, v, do, scale), got, rec = _run(*case, D=D)
    ref = torch_ref(q, k, v, do, causal, window, scale)
    emu = torch_ref(q, k, v, do, causal, window, scale, emulate=True)
    mag = torch_ref(q, k, v, do, causal, window, scale, magnitudes=True)
    for i, name in ((2, "dQ"), (3, "dK"), (4, "dV")):
        assert_close(f"ws {case} {name}", got[i - 2], ref[i], emulated=emu[i], magnitude=mag[i])
    # same math as the recomputing kernels; only fp32 summation order differs
    for i, name in enumerate(("dQ", "dK", "dV")):
        a, r = got[i].float(), rec[i].float()
        assert (a - r).abs().max().item() <= 2e-2 * max(1.0, r.abs().max().item()), name


def test_ws_dq_identical_to_recompute():
    """At head_dim 512 the dQ kernel's result does not depend on whether it also
    stores P / dS (the same kernel runs with and without a workspace)."""
    (_, got, rec) = _run(1, 4, 1, 640, True, 0, torch.bfloat16, seed=3)
    assert torch.equal(got[0], rec[0])


def test_ws_too_small_rejected():
    B, Hq, Hkv, N, D = 1, 2, 1, 256, 512
    q, k, v, do = (t.to(DEV) for t in make_inputs(B, Hq, Hkv, N, D, seed=1))
    o, lse = _fwd(q, k, v, True, 0, 1 / math.sqrt(D), True)
    size = bwd_workspace_size(B, Hq, Hkv, N, D, True, 0)
    ws = torch.empty(size - 256, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        _bwd(q, k, v, o, lse, do, True, 0, 1 / math.sqrt(D), workspace=ws)


def test_default_path_uses_workspace_and_limit_env(monkeypatch):
    """Default full backward at head_dim 512 = materialised path; a zero limit
    selects the recomputing kernels; both agree."""
    B, Hq, Hkv, N, D = 1, 4, 2, 384, 512
    q, k, v, do = (t.to(DEV) for t in make_inputs(B, Hq, Hkv, N, D, seed=5))
    o, lse = _fwd(q, k, v, True, 0, 1 / math.sqrt(D), True)
    a = _bwd(q, k, v, o, lse, do, True, 0, 1 / math.sqrt(D))
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "0")
    r = _bwd(q, k, v, o, lse, do, True, 0, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    assert torch.equal(a[0], r[0])
    for x, y in zip(a[1:], r[1:]):
        assert (x.float() - y.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("D", [256, 512])
def test_workspace_limit_splits_over_kv_heads(monkeypatch, D):
    """A workspace limit below the whole problem's need runs the materialised
    backward over groups of KV heads: bitwise the same gradients."""
    B, Hq, Hkv, N = 2, 8, 4, 384
    q, k, v, do = (t.to(DEV) for t in make_inputs(B, Hq, Hkv, N, D, seed=7))
    scale = 1 / math.sqrt(D)
    o, lse = _fwd(q, k, v, True, 0, scale, True)
    whole = _bwd(q, k, v, o, lse, do, True, 0, scale)
    size = bwd_workspace_size(B, Hq, Hkv, N, D, True, 0)
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", str(size // 3))  # 2 KV heads per chunk
    split = _bwd(q, k, v, o, lse, do, True, 0, scale)
    torch.cuda.synchronize()
    for x, y in zip(whole, split):
        assert torch.equal(x, y)


def test_workspace_split_b1_uneven_kv_groups(monkeypatch):
    """B=1 with H_KV=5 (not a power of two): the split over KV heads starts at
    H_KV // 2 = 2 heads per group, leaving a last group of one; the gradients
    are bitwise those of the whole-workspace run."""
    B, Hq, Hkv, N, D = 1, 10, 5, 320, 512
    q, k, v, do = (t.to(DEV) for t in make_inputs(B, Hq, Hkv, N, D, seed=9))
    scale = 1 / math.sqrt(D)
    o, lse = _fwd(q, k, v, True, 0, scale, True)
    whole = _bwd(q, k, v, o, lse, do, True, 0, scale)
    size = bwd_workspace_size(B, Hq, Hkv, N, D, True, 0)
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", str(2 * (size // Hkv)))  # groups of 2, 2, 1 KV heads
    split = _bwd(q, k, v, o, lse, do, True, 0, scale)
    torch.cuda.synchronize()
    for x, y in zip(whole, split):
        assert torch.equal(x, y)


RECOMPUTE_CASES = [
    # (B, Hq, Hkv, N, D, causal, window, dtype)
    (1, 8, 2, 700, 512, True, 0, torch.bfloat16),
    (2, 4, 4, 257, 512, False, 0, torch.float16),
    (1, 16, 8, 1500, 256, True, 400, torch.float16),
    (1, 4, 1, 513, 256, True, 0, torch.bfloat16),
]


@pytest.mark.parametrize("case", RECOMPUTE_CASES, ids=lambda c: f"B{c[0]}H{c[1]}x{c[2]}N{c[3]}D{c[4]}w{c[6]}")
def test_recompute_backward_matches_fp32(case, monkeypatch):
    """The recomputing backward (gqafa_bwd: dQ + delta, dK, dV kernels), which
    the memory fallback, the row-range entries and the no-alloc entry run,
    held directly to the fp32 reference."""
    B, Hq, Hkv, N, D, causal, window, dt = case
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, 0.5, seed=21, device=DEV)
    scale = 1 / math.sqrt(D)
    o, lse = _fwd(q, k, v, causal, window, scale, True)
    monkeypatch.setenv("GQAFA_BWD_WORKSPACE_LIMIT", "0")
    got = _bwd(q, k, v, o, lse, do, causal, window, scale)
    torch.cuda.synchronize()
    ref = torch_ref(q, k, v, do, causal, window, scale)
    emu = torch_ref(q, k, v, do, causal, window, scale, emulate=True)
    mag = torch_ref(q, k, v, do, causal, window, scale, magnitudes=True)
    for i, name in ((2, "dQ"), (3, "dK"), (4, "dV")):
        assert_close(f"recompute {case} {name}", got[i - 2], ref[i], emulated=emu[i], magnitude=mag[i])


def test_noalloc_backward_matches_fp32():
    """gqafa_bwd_noalloc (delta kept in the library's fixed scratch) held
    directly to the fp32 reference, not only to gqafa_bwd."""
    B, Hq, Hkv, N, D, dt = 1, 8, 2, 600, 512, torch.bfloat16
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, 0.5, seed=31, device=DEV)
    scale = 1 / math.sqrt(D)
    o, lse = _fwd(q, k, v, True, 0, scale, True)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    st = _lib.strides_arg
    _lib.check(_lib.load().gqafa_bwd_noalloc(
        q.data_ptr(), st(q.stride()), k.data_ptr(), st(k.stride()), v.data_ptr(), st(v.stride()),
        o.data_ptr(), st(o.stride()), do.data_ptr(), st(do.stride()), lse.data_ptr(),
        dq.data_ptr(), st(dq.stride()), dk.data_ptr(), st(dk.stride()), dv.data_ptr(), st(dv.stride()),
        B, Hq, Hkv, N, D, scale, 1, 0, _lib.GQAFA_DTYPE_BF16, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = torch_ref(q, k, v, do, True, 0, scale)
    emu = torch_ref(q, k, v, do, True, 0, scale, emulate=True)
    mag = torch_ref(q, k, v, do, True, 0, scale, magnitudes=True)
    for i, name, x in ((2, "dQ", dq), (3, "dK", dk), (4, "dV", dv)):
        assert_close(f"no-alloc {name}", x, ref[i], emulated=emu[i], magnitude=mag[i])


@pytest.mark.parametrize("D,window", [(512, 0), (256, 300), (128, 0)])
def test_partial_backward_writes_fp32_dk_dv(D, window):
    """gqafa_bwd_partial: dK, dV in fp32 (for sums over split query heads),
    which round to exactly the 16-bit outputs of the ordinary backward, with and
    without a workspace."""
    from gemma_triton_flash_attn.attention import _bwd_args

    B, Hq, Hkv, N = 1, 8, 2, 700
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, torch.bfloat16, 0.5, seed=41, device=DEV)
    scale = 1 / math.sqrt(D)
    o, lse = _fwd(q, k, v, True, window, scale, True)
    size = bwd_workspace_size(B, Hq, Hkv, N, D, True, window)
    ref = torch_ref(q, k, v, do, True, window, scale)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for with_ws in ((True, False) if size > 0 else (False,)):
        ws = torch.empty(size, dtype=torch.uint8, device=DEV) if with_ws else None
        dq = torch.empty_like(q)
        dk = torch.empty(k.shape, dtype=torch.float32, device=DEV)
        dv = torch.empty(v.shape, dtype=torch.float32, device=DEV)
        delta = torch.empty(B, Hq, N, device=DEV)
        tail = (ws.data_ptr(), size) if with_ws else (None, 0)
        _lib.check(lib.gqafa_bwd_partial(*_bwd_args(q, k, v, o, do, lse, dq, dk, dv, delta, True, window, scale,
                                                     stream), *tail))
        bufs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty(B, Hq, N, device=DEV))
        if with_ws:
            want = _bwd(q, k, v, o, lse, do, True, window, scale, workspace=torch.empty_like(ws))
        else:
            for st_ in range(3):
                _bwd(q, k, v, o, lse, do, True, window, scale, stage=st_, out=bufs)
            want = bufs[:3]
        torch.cuda.synchronize()
        assert torch.equal(dq, want[0])
        assert torch.equal(dk.to(k.dtype), want[1]) and torch.equal(dv.to(v.dtype), want[2])
        for name, x, r in (("dK", dk, ref[3]), ("dV", dv, ref[4])):
            err = (x - r).abs().max().item()
            assert err <= 2e-2, f"fp32 {name} ws={with_ws}: max-abs {err:.3e}"
