"""The CPU oracle, pinned against fixtures produced by the reference's own
eager attention (tests/golden/make_golden.py). CPU only."""
import os

import numpy as np
import pytest

from helpers import golden_cases, load_golden
from oracle.attention_oracle import attended_pairs, attention_bwd, attention_fwd, attn_flops


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.split("/")[-1][:-4])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_oracle_matches_reference_fixtures(path, dtype):
    c = load_golden(path)
    q, k, v, do = (c[x].float().numpy() for x in ("q", "k", "v", "do"))
    o, lse = attention_fwd(q, k, v, c["causal"], c["slide"], dtype=dtype, chunk=17)
    dq, dk, dv, _ = attention_bwd(q, k, v, o, lse, do, c["causal"], c["slide"], dtype=dtype, chunk=17)
    # The fixtures are fp32 computations of the reference, so agreement is
    # bounded by fp32 rounding in both directions.
    tol = 2e-5
    for name, x in (("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
        ref = c[name].numpy()
        err = np.abs(x - ref).max() / max(1.0, np.abs(ref).max())
        assert err < tol, f"{name}: rel err {err}"


def test_golden_fixture_set_covers_the_cases():
    names = {p.split("/")[-1][:-4] for p in golden_cases()}
    assert {"kernel_d256_swa24", "kernel_d512_causal", "noncausal_window_ignored", "gqa8_swa_ge_n_d32"} <= names


def test_window_ignored_without_causal_and_clamped_at_n():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 2, 20, 8)).astype(np.float32)
    k = rng.standard_normal((1, 1, 20, 8)).astype(np.float32)
    v = rng.standard_normal((1, 1, 20, 8)).astype(np.float32)
    a, _ = attention_fwd(q, k, v, causal=False, window=5)
    b, _ = attention_fwd(q, k, v, causal=False, window=0)
    np.testing.assert_array_equal(a, b)
    c, _ = attention_fwd(q, k, v, causal=True, window=20)
    d, _ = attention_fwd(q, k, v, causal=True, window=0)
    np.testing.assert_array_equal(c, d)


def test_flop_conventions():
    # causal: fwd 2*B*H*N^2*D, fwd+bwd 7*B*H*N^2*D (reference convention)
    assert attn_flops(1, 32, 16384, 512, True) == 2 * 32 * 16384 ** 2 * 512
    assert attn_flops(1, 32, 16384, 512, True, bwd=True) == 7 * 32 * 16384 ** 2 * 512
    # sliding window W < N: P = N*W - W(W-1)/2
    assert attended_pairs(4096, True, 1024) == 4096 * 1024 - 1024 * 1023 // 2
    assert attended_pairs(512, True, 1024) == 512 * 512 // 2
    assert attended_pairs(100, False, 7) == 100 * 100


# ---------------------------------------------------------------- eager CPU path
# oracle/eager_ref.py restates the reference's eager attention_gqa_ref /
# attention_swa_ref (flash_attn/attention.py:611-642): the CPU path that
# bench.py times as the reference arm. It is pinned to the same fixtures and,
# where a checkout of the reference is present, to the reference module itself.
REF_ROOT = os.environ.get("GQAFA_REFERENCE_ROOT", "/root/reference")


def _eager_run(c):
    import torch

    from oracle.eager_ref import sdpa_gqa

    q, k, v = (c[x].float().requires_grad_(True) for x in ("q", "k", "v"))
    o = sdpa_gqa(q, k, v, c["causal"], c["slide"])
    o.backward(c["do"].float())
    return o.detach(), q.grad, k.grad, v.grad


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.split("/")[-1][:-4])
def test_eager_restatement_matches_reference_fixtures(path):
    c = load_golden(path)
    o, dq, dk, dv = _eager_run(c)
    for name, x in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        ref = c[name]
        err = (x - ref).abs().max().item() / max(1.0, ref.abs().max().item())
        assert err < 1e-5, f"{name}: rel err {err}"


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_ROOT, "flash_attn")), reason="no reference checkout")
@pytest.mark.parametrize("causal", [True, False])
def test_eager_restatement_is_the_reference_function(causal):
    """Config-1-shaped (smaller N) fp32 inputs: bitwise equal to the reference's
    own attention_gqa_ref, forward and autograd backward."""
    import importlib.util

    import torch

    from oracle.eager_ref import sdpa_gqa

    spec = importlib.util.spec_from_file_location("_ref_attention", os.path.join(REF_ROOT, "flash_attn", "attention.py"))
    try:
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # the module imports triton at top level
        pytest.skip(f"reference module not importable here: {e}")
    g = torch.Generator().manual_seed(7)
    q, k, v, do = (torch.randn(s, generator=g) for s in ((1, 8, 64, 32), (1, 2, 64, 32), (1, 2, 64, 32), (1, 8, 64, 32)))
    outs = []
    for fn in (mod.attention_gqa_ref, lambda a, b, c_, causal: sdpa_gqa(a, b, c_, causal)):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = fn(qq, kk, vv, causal=causal)
        o.backward(do)
        outs.append((o.detach(), qq.grad, kk.grad, vv.grad))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
