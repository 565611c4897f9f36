"""Parity of the sm_100a kernels (through the C ABI) against the reference's
math: the golden fixtures made by the reference's own eager code, the CPU
oracle, and an fp32 PyTorch computation for sizes the oracle is too slow for.

Criterion: O, dQ, dK, dV within max-abs 2e-2 and fp32
cosine >= 0.9999 of an fp32 computation on the same (16-bit) inputs; LSE within
1e-3."""
import math

import numpy as np
import pytest
import torch

import gemma_triton_flash_attn as gfa
from gemma_triton_flash_attn import _lib
from gemma_triton_flash_attn.attention import flash_attn_gqa_backward, flash_attn_gqa_forward_with_lse
from helpers import ATOL, LSE_ATOL, assert_close, golden_cases, load_golden, make_inputs, metrics, torch_ref
from oracle.attention_oracle import attention_bwd, attention_fwd

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert _lib.device_status(torch.cuda.current_device(), reset=True) == 0, "a kernel wait timed out"


def run_both(q, k, v, do, causal, slide, scale=None):
    o, lse = flash_attn_gqa_forward_with_lse(q, k, v, causal, slide, scale)
    dq, dk, dv = flash_attn_gqa_backward(q, k, v, o, lse, do, causal, slide, scale)
    torch.cuda.synchronize()
    return o, lse, dq, dk, dv


def check_all(got, ref, tag="", emulated=None, magnitudes=None):
    names = ("O", "LSE", "dQ", "dK", "dV")
    for i, (name, x, r) in enumerate(zip(names, got, ref)):
        if name == "LSE":
            assert torch.isfinite(x).all()
            err = (x.float().cpu() - r.float().cpu()).abs().max().item()
            assert err <= LSE_ATOL, f"{tag} LSE max-abs {err:.3e}"
        else:
            assert_close(f"{tag} {name}", x, r, emulated=None if emulated is None else emulated[i],
                         magnitude=None if magnitudes is None else magnitudes[i])


def ref_set(q, k, v, do, causal, slide, scale=None):
    """(pure fp32 reference, fp32 with the algorithm's 16-bit roundings, magnitudes)."""
    return (torch_ref(q, k, v, do, causal, slide, scale),
            torch_ref(q, k, v, do, causal, slide, scale, emulate=True),
            torch_ref(q, k, v, do, causal, slide, scale, magnitudes=True))


# ----------------------------------------------------------------- golden
# every fixture whose head_dim the kernels implement (64, 128, 256, 512)
KERNEL_GOLDEN = [p for p in golden_cases() if int(np.load(p)["meta"][4]) in (64, 128, 256, 512)]


@pytest.mark.parametrize("path", KERNEL_GOLDEN, ids=lambda p: p.split("/")[-1][:-4])
def test_kernel_matches_reference_golden(path):
    c = load_golden(path)
    q, k, v, do = (c[x].to(DEV) for x in ("q", "k", "v", "do"))
    got = run_both(q, k, v, do, c["causal"], c["slide"])
    check_all(got, [c[x] for x in ("o", "lse", "dq", "dk", "dv")], tag=path.split("/")[-1])


# ----------------------------------------------------------------- oracle (CPU numpy)
def test_config1_shape_against_cpu_oracle():
    # BASELINE config 1 shape (B1, 32/4, N512, D512, causal) with bf16 inputs.
    q, k, v, do = make_inputs(1, 32, 4, 512, 512, torch.bfloat16, factor=1.0, seed=11)
    o, lse = attention_fwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), True, 0)
    dq, dk, dv, _ = attention_bwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), o, lse,
                                  do.float().numpy(), True, 0)
    got = run_both(q.to(DEV), k.to(DEV), v.to(DEV), do.to(DEV), True, 0)
    emu = torch_ref(q.to(DEV), k.to(DEV), v.to(DEV), do.to(DEV), True, 0, emulate=True)
    mag = torch_ref(q.to(DEV), k.to(DEV), v.to(DEV), do.to(DEV), True, 0, magnitudes=True)
    check_all(got, [torch.from_numpy(x) for x in (o, lse, dq, dk, dv)], tag="config1", emulated=emu,
              magnitudes=mag)


# ----------------------------------------------------------------- BASELINE config shapes (fp32 torch)
CONFIGS = [
    # name, B, Hq, Hkv, N, D, causal, slide, dtype, factor
    ("cfg2_bf16_1k", 1, 32, 4, 1024, 512, True, 0, torch.bfloat16, 0.5),
    ("cfg2_fp16_2k", 1, 32, 4, 2048, 512, True, 0, torch.float16, 0.5),
    ("cfg2_bf16_4k", 1, 32, 4, 4096, 512, True, 0, torch.bfloat16, 0.5),
    ("cfg3_fp16_1k", 1, 16, 8, 1024, 256, True, 1024, torch.float16, 1.0),
    ("cfg3_fp16_4k", 1, 16, 8, 4096, 256, True, 1024, torch.float16, 1.0),
    ("cfg4_bf16_1k", 4, 16, 2, 1024, 512, True, 0, torch.bfloat16, 1.0),
    ("cfg5_sliding_bf16", 2, 16, 8, 2048, 256, True, 512, torch.bfloat16, 1.0),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: c[0])
def test_baseline_config_shapes(cfg):
    name, B, Hq, Hkv, N, D, causal, slide, dt, fac = cfg
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, fac, seed=5, device=DEV)
    ref, emu, mag = ref_set(q, k, v, do, causal, slide)
    check_all(run_both(q, k, v, do, causal, slide), ref, tag=name, emulated=emu, magnitudes=mag)


# ----------------------------------------------------------------- edge cases
EDGE = []
for D in (256, 512):
    for N in (1, 7, 64, 65, 127, 129, 200):
        EDGE.append((1, 4, 2, N, D, True, 0))
    EDGE += [
        (1, 2, 1, 100, D, False, 0),      # non-causal, ragged
        (1, 2, 2, 130, D, True, 1),       # window 1: diagonal only
        (1, 2, 1, 131, D, True, 3),
        (1, 4, 1, 96, D, True, 96),       # window == N  -> causal
        (1, 4, 1, 96, D, True, 95),       # window == N - 1
        (1, 4, 1, 96, D, True, 97),       # window > N
        (1, 4, 1, 80, D, False, 16),      # window ignored without causal
        (3, 16, 1, 70, D, True, 0),       # GQA 16:1, B=3
        (2, 8, 8, 150, D, True, 40),      # MHA with window
        (2, 4, 2, 200, D, True, 0),       # last tile partly past N with two items only:
        (1, 2, 1, 193, D, False, 0),      # exposed an early epilogue (accumulator not yet final)
    ]


@pytest.mark.parametrize("case", EDGE, ids=lambda c: "B{}_H{}-{}_N{}_D{}_c{}_w{}".format(*c))
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_edge_cases(case, dt):
    B, Hq, Hkv, N, D, causal, slide = case
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, 1.0, seed=N + D, device=DEV)
    ref, emu, mag = ref_set(q, k, v, do, causal, slide)
    check_all(run_both(q, k, v, do, causal, slide), ref, tag=str(case), emulated=emu, magnitudes=mag)


def test_hf_layout_strided_inputs_need_no_copy():
    # HF gives (B, N, H, D) storage viewed as (B, H, N, D).
    B, Hq, Hkv, N, D = 2, 8, 2, 300, 256
    g = torch.Generator().manual_seed(9)
    qs = torch.randn(B, N, Hq, D, generator=g).bfloat16().to(DEV)
    ks = torch.randn(B, N, Hkv, D, generator=g).bfloat16().to(DEV)
    vs = torch.randn(B, N, Hkv, D, generator=g).bfloat16().to(DEV)
    dos = torch.randn(B, N, Hq, D, generator=g).bfloat16().to(DEV)
    q, k, v, do = (t.transpose(1, 2) for t in (qs, ks, vs, dos))
    assert not q.is_contiguous()
    got = run_both(q, k, v, do, True, 64)
    assert got[0].stride() == q.stride(), "O keeps the (B, N, H, D) storage of q"
    ref = run_both(*(t.contiguous() for t in (q, k, v, do)), True, 64)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_deterministic_bitwise():
    q, k, v, do = make_inputs(1, 8, 2, 700, 512, torch.bfloat16, 0.5, seed=21, device=DEV)
    a = run_both(q, k, v, do, True, 0)
    b = run_both(q, k, v, do, True, 0)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_custom_softmax_scale():
    q, k, v, do = make_inputs(1, 4, 2, 256, 256, torch.bfloat16, 0.25, seed=2, device=DEV)
    ref = torch_ref(q, k, v, do, True, 0, scale=1.0)
    check_all(run_both(q, k, v, do, True, 0, scale=1.0), ref, tag="scale=1")


def test_autograd_function_and_inference_path():
    q, k, v, do = make_inputs(1, 8, 2, 384, 512, torch.bfloat16, 0.5, seed=4, device=DEV)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    out = gfa.flash_attn_gqa_train(qg, kg, vg, causal=True, slide_size=0)
    out.backward(do)
    ro, rl, rdq, rdk, rdv = torch_ref(q, k, v, do, True, 0)
    assert_close("train O", out, ro)
    assert_close("train dQ", qg.grad, rdq)
    assert_close("train dK", kg.grad, rdk)
    assert_close("train dV", vg.grad, rdv)
    assert qg.grad.dtype == torch.bfloat16
    inf = gfa.attention_flash_gqa(q, k, v, causal=True, slide_size=0, BLOCK_Q=64, num_warps=4)
    assert torch.equal(inf, out.detach())


def test_validation_errors_on_gpu():
    q, k, v, _ = make_inputs(1, 4, 2, 64, 256, torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="self-attention"):
        gfa.flash_attn_gqa_train(q, k[:, :, :32], v[:, :, :32], causal=True)
    with pytest.raises(ValueError, match="multiple of H_KV"):
        gfa.flash_attn_gqa_train(q[:, :3], k, v)
    with pytest.raises(NotImplementedError):
        gfa.flash_attn_gqa_train(q[..., :96].contiguous(), k[..., :96].contiguous(), v[..., :96].contiguous())
    with pytest.raises(NotImplementedError):
        gfa.flash_attn_gqa_train(q.float(), k.float(), v.float())


# ----------------------------------------------------------------- full-size properties
def test_full_size_config2_properties():
    """Config 2 at N=16K: sampled rows of O / LSE / dQ against fp32, and the
    size-independent identities sum_kv dV = sum_q dO (rows of P sum to 1) and
    sum_kv dK = 0 (rows of dS sum to 0) per KV group."""
    B, Hq, Hkv, N, D = 1, 32, 4, 16384, 512
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, torch.bfloat16, 0.5, seed=77, device=DEV)
    o, lse, dq, dk, dv = run_both(q, k, v, do, True, 0)
    G = Hq // Hkv
    rows = torch.cat([torch.arange(0, 64), torch.arange(8000, 8064), torch.arange(N - 128, N)]).to(DEV)
    for h in (0, 13, 31):
        kv = h // G
        qs = q[:, h:h + 1, rows].float()
        s = (qs @ k[:, kv:kv + 1].float().transpose(-1, -2)) / math.sqrt(D)
        mask = torch.arange(N, device=DEV)[None, :] <= rows[:, None]
        s = s.masked_fill(~mask, float("-inf"))
        l = torch.logsumexp(s, -1)
        p = torch.exp(s - l[..., None])
        ro = p @ v[:, kv:kv + 1].float()
        dos = do[:, h:h + 1, rows].float()
        dp = dos @ v[:, kv:kv + 1].float().transpose(-1, -2)
        delta = (dos * ro).sum(-1, keepdim=True)
        rdq = ((p * (dp - delta)) @ k[:, kv:kv + 1].float()) / math.sqrt(D)
        assert_close(f"O rows h{h}", o[:, h:h + 1, rows], ro)
        assert (lse[:, h:h + 1, rows] - l).abs().max().item() <= LSE_ATOL
        assert_close(f"dQ rows h{h}", dq[:, h:h + 1, rows], rdq)
    dv_sum = dv.float().sum(2)                                  # (B, Hkv, D)
    do_sum = do.float().view(B, Hkv, G, N, D).sum((2, 3))
    rel = ((dv_sum - do_sum).norm() / do_sum.norm()).item()
    assert rel < 2e-3, rel
    # sum_kv dS = 0 holds exactly for the fp32 math; the residual here comes from
    # delta being formed from the bf16-stored O and dS being rounded to bf16.
    dk_sum = dk.float().sum(2)
    assert (dk_sum.norm() / dk.float().norm()).item() < 1e-2


def test_full_size_config3_swa_properties():
    B, Hq, Hkv, N, D, W = 1, 16, 8, 32768, 256, 1024
    q, k, v, do = make_inputs(B, Hq, Hkv, N, D, torch.float16, 1.0, seed=78, device=DEV)
    o, lse, dq, dk, dv = run_both(q, k, v, do, True, W)
    # sampled rows against fp32 restricted to their window
    for r0 in (0, 5000, N - 64):
        rows = slice(r0, r0 + 64)
        k0 = max(0, r0 - W + 1)
        sub = [t[:, :, k0:r0 + 64] for t in (q, k, v, do)]
        ro, rl, rdq, _, _ = torch_ref(*sub, True, W)
        off = r0 - k0
        assert_close(f"SWA O rows {r0}", o[:, :, rows], ro[:, :, off:off + 64])
        assert (lse[:, :, rows] - rl[:, :, off:off + 64]).abs().max().item() <= LSE_ATOL
        assert_close(f"SWA dQ rows {r0}", dq[:, :, rows], rdq[:, :, off:off + 64])
    G = Hq // Hkv
    dv_sum = dv.float().sum(2)
    do_sum = do.float().view(B, Hkv, G, N, D).sum((2, 3))
    assert ((dv_sum - do_sum).norm() / do_sum.norm()).item() < 2e-3


def test_short_tiles_repeated():
    """Tiles with one or two column items finish their elementwise work
    quickly; the epilogue must still wait for the last accumulate MMA. Run the
    shapes that exposed an early read several times."""
    for rep in range(5):
        for (B, Hq, Hkv, N, D, causal) in ((2, 4, 2, 200, 512, True), (1, 2, 1, 193, 512, False),
                                           (1, 4, 2, 130, 256, True), (2, 2, 1, 129, 512, True)):
            q, k, v, do = make_inputs(B, Hq, Hkv, N, D, torch.bfloat16, 0.5, seed=rep, device=DEV)
            ref = torch_ref(q, k, v, do, causal, 0)
            check_all(run_both(q, k, v, do, causal, 0), ref, tag=f"rep{rep} N{N} D{D}")
