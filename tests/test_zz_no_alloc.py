"""gqafa_bwd_noalloc: the backward entry point for callers that cannot
allocate device memory (they hold only their input and output tensors, e.g.
behind an FFI, or run with all device memory planned in advance and may not
call cudaMalloc). It keeps the per-row delta workspace in a fixed array inside
the library. This file is collected last on purpose: it must pass both alone
in a fresh process and after every other test."""
import math

import pytest
import torch

from gemma_triton_flash_attn import _lib
from gemma_triton_flash_attn.attention import flash_attn_gqa_forward_with_lse
from helpers import assert_close, make_inputs

pytestmark = pytest.mark.gpu

DT = {torch.bfloat16: _lib.GQAFA_DTYPE_BF16, torch.float16: _lib.GQAFA_DTYPE_FP16}


def _grads(entry, q, k, v, o, lse, do, causal, window, with_delta):
    B, Hq, N, D = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    st = _lib.strides_arg
    args = [q.data_ptr(), st(q.stride()), k.data_ptr(), st(k.stride()), v.data_ptr(), st(v.stride()),
            o.data_ptr(), st(o.stride()), do.data_ptr(), st(do.stride()), lse.data_ptr(),
            dq.data_ptr(), st(dq.stride()), dk.data_ptr(), st(dk.stride()), dv.data_ptr(), st(dv.stride())]
    if with_delta:
        delta = torch.empty((B, Hq, N), dtype=torch.float32, device=q.device)
        args.append(delta.data_ptr())
    args += [B, Hq, k.shape[1], N, D, 1.0 / math.sqrt(D), int(causal), window, DT[q.dtype],
             torch.cuda.current_stream().cuda_stream]
    _lib.check(entry(*args))
    return dq, dk, dv


@pytest.mark.parametrize("shape", [
    # B, H_Q, H_KV, N, D, causal, window, dtype
    (2, 8, 2, 300, 512, True, 0, torch.bfloat16),
    (1, 16, 8, 1100, 256, True, 256, torch.float16),
], ids=["d512_causal_bf16", "d256_swa_fp16"])
def test_noalloc_backward_matches_allocating_entry_point(shape):
    B, Hq, Hkv, N, D, causal, window, dt = shape
    lib = _lib.load()
    for call in range(2):  # two calls in a row: the shared scratch keeps the last call's contents
        q, k, v, do = make_inputs(B, Hq, Hkv, N, D, dt, 0.5, seed=100 + call, device="cuda")
        o, lse = flash_attn_gqa_forward_with_lse(q, k, v, causal, window)
        want = _grads(lib.gqafa_bwd, q, k, v, o, lse, do, causal, window, with_delta=True)
        got = _grads(lib.gqafa_bwd_noalloc, q, k, v, o, lse, do, causal, window, with_delta=False)
        torch.cuda.synchronize()
        assert _lib.device_status(torch.cuda.current_device()) == 0
        for name, a, b in zip(("dQ", "dK", "dV"), got, want):
            assert_close(f"no-alloc {name} call {call}", a, b.float())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    B, Hq, Hkv, N, D = 1, 64, 8, 32768, 256  # B*H_Q*N = 2^21 > 2^20 rows
    st = _lib.strides_arg((Hq * N * D, N * D, D, 1))
    kst = _lib.strides_arg((Hkv * N * D, N * D, D, 1))
    f = 0x100000  # never dereferenced: the size check comes first
    rc = lib.gqafa_bwd_noalloc(f, st, f, kst, f, kst, f, st, f, st, f, f, st, f, kst, f, kst,
                               B, Hq, Hkv, N, D, 0.0625, 1, 0, 1, None)
    assert rc == _lib.GQAFA_ERR_INVALID
    assert "exceeds the fixed scratch" in lib.gqafa_last_error().decode()
