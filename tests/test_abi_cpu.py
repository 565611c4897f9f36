"""The C-ABI library loads, exports every declared symbol and validates its
arguments on the host. No GPU needed: every call below fails validation
before any CUDA work."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from gemma_triton_flash_attn import _lib

HEADER = os.path.join(ROOT, "include", "gqa_fa_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"GQAFA_API\s+[\w\s\*]+?\b(gqafa_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)
    for n in names:
        assert hasattr(lib, n), n


def test_library_is_in_tree_and_built_for_sm100a():
    assert os.path.commonpath([_lib.LIB_PATH, ROOT]) == ROOT
    # the build recipe targets sm_100a only (the version string says the same)
    make = open(os.path.join(ROOT, "gemma-triton-flash-attn_b200", "Makefile")).read()
    arch = re.findall(r"^ARCH\s*:=\s*(.*)$", make, re.M)
    assert arch == ["-gencode arch=compute_100a,code=sm_100a"], arch
    assert "sm_100a" in _lib.version()


def test_supported_and_version():
    lib = _lib.load()
    assert lib.gqafa_supported(512, 1) == 1 and lib.gqafa_supported(256, 0) == 1
    assert lib.gqafa_supported(128, 1) == 1 and lib.gqafa_supported(64, 0) == 1
    assert lib.gqafa_supported(96, 1) == 0 and lib.gqafa_supported(32, 1) == 0 and lib.gqafa_supported(512, 7) == 0
    assert "sm_100a" in _lib.version()


def _fwd(**over):
    lib = _lib.load()
    st = _lib.strides_arg((32 * 64 * 512, 64 * 512, 512, 1))
    kst = _lib.strides_arg((4 * 64 * 512, 64 * 512, 512, 1))
    fake = 0x100000  # never dereferenced: validation fails first
    args = dict(q=fake, qs=st, k=fake, ks=kst, v=fake, vs=kst, o=fake, os=st, lse=None,
                B=1, Hq=32, Hkv=4, N=64, D=512, scale=0.044, causal=1, window=0, dtype=1)
    args.update(over)
    return lib.gqafa_fwd(args["q"], args["qs"], args["k"], args["ks"], args["v"], args["vs"],
                         args["o"], args["os"], args["lse"], args["B"], args["Hq"], args["Hkv"],
                         args["N"], args["D"], args["scale"], args["causal"], args["window"],
                         args["dtype"], None)


@pytest.mark.parametrize("over,code,msg", [
    (dict(Hq=30), _lib.GQAFA_ERR_INVALID, "multiple of H_KV"),
    (dict(D=96), _lib.GQAFA_ERR_UNSUPPORTED, "head_dim 96"),
    (dict(dtype=3), _lib.GQAFA_ERR_INVALID, "dtype"),
    (dict(N=0), _lib.GQAFA_ERR_INVALID, "positive"),
    (dict(scale=0.0), _lib.GQAFA_ERR_INVALID, "softmax_scale"),
    (dict(window=-1), _lib.GQAFA_ERR_INVALID, "window"),
    (dict(q=None), _lib.GQAFA_ERR_INVALID, "null pointer"),
    (dict(q=0x100008), _lib.GQAFA_ERR_INVALID, "16-byte aligned"),
    (dict(qs=_lib.strides_arg((32 * 64 * 512, 64 * 512, 1, 64))), _lib.GQAFA_ERR_INVALID, "last (head_dim) stride"),
    (dict(qs=_lib.strides_arg((32 * 64 * 512, 64 * 512, 516, 1))), _lib.GQAFA_ERR_INVALID, "multiples of 8"),
])
def test_fwd_validation(over, code, msg):
    rc = _fwd(**over)
    assert rc == code
    assert msg in _lib.load().gqafa_last_error().decode()


def test_check_maps_codes_to_python_exceptions():
    assert _fwd(D=96) == _lib.GQAFA_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.GQAFA_ERR_UNSUPPORTED)
    assert _fwd(Hq=30) == _lib.GQAFA_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(_lib.GQAFA_ERR_INVALID)


def test_bwd_validation_requires_lse_and_delta():
    lib = _lib.load()
    st = _lib.strides_arg((8 * 64 * 256, 64 * 256, 256, 1))
    f = 0x100000
    rc = lib.gqafa_bwd(f, st, f, st, f, st, f, st, f, st, None, f, st, f, st, f, st, None,
                       1, 8, 8, 64, 256, 0.0625, 1, 0, 0, None)
    assert rc == _lib.GQAFA_ERR_INVALID
    assert "lse and delta" in lib.gqafa_last_error().decode()


def _blocks_per_head(n, causal, window):
    """Attended (128-query tile, 256-key block) pairs of one head, counted directly."""
    total = 0
    for t in range((n + 127) // 128):
        hi = min(n, 128 * t + 128) if causal else n
        lo = max(0, 128 * t - window + 1) if (causal and window) else 0
        total += (hi + 255) // 256 - lo // 256
    return total


@pytest.mark.parametrize("n,causal,window", [(16384, True, 0), (300, True, 0), (129, True, 0), (200, False, 0),
                                             (1000, True, 300), (777, True, 129), (64, False, 0),
                                             (5000, True, 5000), (4096, True, 1)])
def test_bwd_workspace_size(n, causal, window):
    lib = _lib.load()
    w = window if (causal and 0 < window < n) else 0
    want = 2 * 2 * 8 * _blocks_per_head(n, causal, w) * 128 * 256 * 2
    assert lib.gqafa_bwd_workspace_size(2, 8, 2, n, 512, int(causal), window) == want
    assert lib.gqafa_bwd_workspace_size(2, 8, 2, n, 256, int(causal), window) == want
    assert lib.gqafa_bwd_workspace_size(2, 8, 2, n, 128, int(causal), window) == 0  # recomputing backward
    assert lib.gqafa_bwd_workspace_size(2, 8, 2, n, 96, int(causal), window) == -1
    assert lib.gqafa_bwd_workspace_size(2, 8, 3, n, 512, int(causal), window) == -1


def test_torch_operators_load_and_propagate_shapes():
    """libgqa_fa_ops.so registers torch.ops.gqafa.fwd / bwd over the C ABI;
    their Meta kernels give the output shapes without a GPU."""
    import torch

    ops = _lib.ops()
    q = torch.empty(2, 8, 100, 512, device="meta", dtype=torch.bfloat16)
    k = torch.empty(2, 2, 100, 512, device="meta", dtype=torch.bfloat16)
    o, lse = ops.fwd(q, k, k, True, 0, 512 ** -0.5, True)
    assert o.shape == q.shape and o.dtype == q.dtype and lse.shape == (2, 8, 100) and lse.dtype == torch.float32
    dq, dk, dv = ops.bwd(q, k, k, o, lse, q, True, 0, 512 ** -0.5, None)
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == k.shape
    assert "Tensor? workspace" in str(ops.bwd.default._schema)
