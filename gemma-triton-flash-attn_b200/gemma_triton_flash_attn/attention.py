"""GQA flash attention for Gemma-4 shapes on B200 (sm_100a).

Host-side mirror of the reference module ``flash_attn/attention.py``
(zzhhjjj/gemma-triton-flash-attn): the same public names, argument meaning and
return values, with every launch going through the C ABI of
``libgqa_fa_b200.so`` (include/gqa_fa_b200.h) instead of Triton.

Public API (reference line numbers in flash_attn/attention.py):
    attention_flash_gqa(q, k, v, causal=False, slide_size=0, ...)   :540-604
    flash_attn_gqa_train(q, k, v, causal=False, slide_size=0)       :1625-1635
    FlashAttnGQAFunction.apply(q, k, v, causal, slide_size)         :1433-1622
    attention_gqa_ref(q, k, v, causal=False)                         :611-619
    attention_swa_ref(q, k, v, slide_size)                           :622-642
    attention(q, k, v)                                               :11-17

Shapes: q (B, H_Q, N, D); k, v (B, H_KV, N, D); H_Q a multiple of H_KV; fp16
or bf16; D in {256, 512}. ``slide_size > 0`` applies a causal sliding window
(query i sees keys i-slide_size+1 .. i) and is ignored when ``causal`` is
False, exactly as in the reference.

Differences from the reference, all deliberate:
  * Validation: CPU tensors, mismatched devices/dtypes, H_Q % H_KV != 0 and a
    key length different from the query length raise instead of silently
    reading the wrong range (reference: attention.py:552-553, :272).
  * The tile-size keyword arguments of ``attention_flash_gqa`` are accepted and
    ignored: tiles are fixed per head_dim in the CUDA library.
  * ``FlashAttnGQAFunction.apply`` takes an optional 6th argument
    ``softmax_scale`` (default 1/sqrt(D), the reference's fixed value).
"""
from __future__ import annotations

import math
import os

import torch

from . import _lib

__all__ = [
    "attention_flash_gqa",
    "flash_attn_gqa_train",
    "FlashAttnGQAFunction",
    "attention_gqa_ref",
    "attention_swa_ref",
    "attention",
]


# --------------------------------------------------------------------------
# PyTorch references (the reference's own eager definitions of the math)
# --------------------------------------------------------------------------

def attention(q, k, v):
    """Standard scaled dot-product attention, (B, H, N, D) in and out."""
    return torch.nn.functional.scaled_dot_product_attention(q, k, v)


def _expand_kv(q, k, v):
    h_q, h_kv = q.shape[1], k.shape[1]
    if h_q != h_kv:
        g = h_q // h_kv
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
    return k, v


def attention_gqa_ref(q, k, v, causal=False):
    """SDPA reference for GQA: KV heads repeated to the query head count."""
    k, v = _expand_kv(q, k, v)
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)


def attention_swa_ref(q, k, v, slide_size):
    """SDPA reference for causal sliding-window GQA with an explicit (N, N) mask.

    Query i attends key j iff j <= i and i - j < slide_size. Small N only.
    """
    k, v = _expand_kv(q, k, v)
    n = q.shape[2]
    pos = torch.arange(n, device=q.device)
    allowed = (pos[None, :] <= pos[:, None]) & ((pos[:, None] - pos[None, :]) < slide_size)
    bias = torch.zeros(n, n, dtype=q.dtype, device=q.device)
    bias = bias.masked_fill(~allowed, float("-inf"))
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=bias[None, None])


# --------------------------------------------------------------------------
# Launch helpers
# --------------------------------------------------------------------------

_DTYPES = {torch.float16: _lib.GQAFA_DTYPE_FP16, torch.bfloat16: _lib.GQAFA_DTYPE_BF16}


def _abi_ready(t: torch.Tensor) -> torch.Tensor:
    """Return `t` if its layout is TMA-legal, else a contiguous copy.

    Legal: last stride 1, other strides multiples of 8 elements, 16-byte
    aligned data pointer. HF's transposed (B, N, H, D) views qualify.
    """
    st = t.stride()
    ok = (
        st[3] == 1
        and t.data_ptr() % 16 == 0
        and all((s % 8 == 0) or (n == 1) for s, n in zip(st[:3], t.shape[:3]))
    )
    return t if ok else t.contiguous()


def _check_inputs(q, k, v, kv_cache=False, causal=False):
    """Validate q, k, v. kv_cache=True accepts a key length different from the
    query length (forward only): with causal attention the queries are the
    last positions of the keys, so the key length must not be shorter."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D (B, H, N, D), got shape {tuple(t.shape)}")
        if not t.is_cuda:
            raise RuntimeError(
                f"{name} is on {t.device}: gemma_triton_flash_attn runs only on CUDA (sm_100a); "
                "there is no CPU fallback"
            )
    if not (q.device == k.device == v.device):
        raise ValueError(f"q, k, v must share a device, got {q.device}, {k.device}, {v.device}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v must share a dtype, got {q.dtype}, {k.dtype}, {v.dtype}")
    if q.dtype not in _DTYPES:
        raise NotImplementedError(f"dtype {q.dtype} is not supported (fp16, bf16)")
    b, h_q, n, d = q.shape
    if k.shape != v.shape:
        raise ValueError(f"k and v shapes differ: {tuple(k.shape)} vs {tuple(v.shape)}")
    if k.shape[0] != b or k.shape[3] != d:
        raise ValueError(f"k/v shape {tuple(k.shape)} incompatible with q {tuple(q.shape)}")
    if k.shape[2] != n and not kv_cache:
        raise ValueError(
            f"key length {k.shape[2]} != query length {n}: only self-attention is supported here "
            "(attention_flash_gqa takes a longer KV cache)"
        )
    if kv_cache and causal and k.shape[2] < n:
        raise ValueError(f"causal attention needs key length {k.shape[2]} >= query length {n}")
    h_kv = k.shape[1]
    if h_q % h_kv != 0:
        raise ValueError(f"H_Q ({h_q}) must be a multiple of H_KV ({h_kv})")


def _normalize_window(causal: bool, slide_size, n: int) -> int:
    slide = int(slide_size) if slide_size else 0
    if slide < 0:
        raise ValueError("slide_size must be >= 0")
    # Reference: a window covering the whole sequence is plain causal, and the
    # window is only applied with causal=True (attention.py:558-559, :289).
    if not causal or slide >= n:
        return 0
    return slide


class _DeviceScope:
    """Make `device` current for the duration of a call (cheap when it already is)."""

    __slots__ = ("dev", "prev")

    def __init__(self, device: torch.device):
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def _fwd(q, k, v, causal, window, scale, want_lse, rows=None, out=None):
    """Forward launch. `rows` = (begin, end) computes only those query rows,
    into the preallocated `out` = (o, lse) (sequence-split multi-GPU path).
    A key length different from the query length runs gqafa_fwd_kv."""
    lib = _lib.load()
    b, h_q, n, d = q.shape
    h_kv, nk = k.shape[1], k.shape[2]
    if out is None and rows is None:
        # the hot path: one torch operator call (torch_ops.cpp) over the C ABI
        o, lse = _lib.ops().fwd(q, k, v, bool(causal), int(window), float(scale), bool(want_lse))
        return o, (lse if want_lse else None)
    q, k, v = _abi_ready(q), _abi_ready(k), _abi_ready(v)
    if out is None:
        o = torch.empty_like(q)  # keeps q's layout (e.g. HF's (B, N, H, D) storage)
        o = _abi_ready(o)
        lse = torch.empty((b, h_q, n), dtype=torch.float32, device=q.device) if want_lse else None
    else:
        o, lse = out
    if nk != n:
        if rows is not None:
            raise ValueError("row ranges need key length == query length")
        fn = lambda *a: lib.gqafa_fwd_kv(*a[:13], nk, *a[13:])  # noqa: E731
    elif rows is None:
        fn = lib.gqafa_fwd
    else:
        fn = lambda *a: lib.gqafa_fwd_rows(*a, int(rows[0]), int(rows[1]))  # noqa: E731
    with _DeviceScope(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = fn(
            q.data_ptr(), _lib.strides_arg(q.stride()),
            k.data_ptr(), _lib.strides_arg(k.stride()),
            v.data_ptr(), _lib.strides_arg(v.stride()),
            o.data_ptr(), _lib.strides_arg(o.stride()),
            lse.data_ptr() if lse is not None else None,
            b, h_q, h_kv, n, d, float(scale), 1 if causal else 0, int(window),
            _DTYPES[q.dtype], stream,
        )
    _lib.check(rc)
    return o, lse


def _workspace_limit(device=None):
    """Largest backward workspace (bytes) `_bwd` may allocate.

    GQAFA_BWD_WORKSPACE_LIMIT (bytes) overrides; 0 turns the materialised
    backward off. Otherwise the budget is GQAFA_BWD_WORKSPACE_FRACTION
    (default 0.5) of the device memory that is free right now: free in the
    driver plus what torch's caching allocator holds unused. A workspace over
    the budget makes the backward run over groups of KV heads (each group's
    share within the budget), and the recomputing backward (no workspace) when
    one KV head's share is over it too. A workspace that the caching allocator
    can serve from memory it already holds unused is always allowed (it adds
    nothing to the process's footprint)."""
    env = os.environ.get("GQAFA_BWD_WORKSPACE_LIMIT")
    if env is not None:
        return int(env)
    if device is None:
        return None
    frac = float(os.environ.get("GQAFA_BWD_WORKSPACE_FRACTION", "0.5"))
    free, _ = torch.cuda.mem_get_info(device)
    cached = torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    return int(frac * (free + cached))


def bwd_workspace_size(b, h_q, h_kv, n, d, causal, window):
    """Bytes of workspace the materialised backward needs (0: not applicable)."""
    size = _lib.load().gqafa_bwd_workspace_size(b, h_q, h_kv, n, d, 1 if causal else 0, int(window))
    if size < 0:
        _lib.check(_lib.GQAFA_ERR_INVALID)
    return int(size)


def _alloc_workspace(size, device):
    if size <= 0:
        return None
    env = os.environ.get("GQAFA_BWD_WORKSPACE_LIMIT")
    if env is not None:
        if size > int(env):
            return None
    elif size > torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device):
        # Memory the caching allocator already holds unused (the previous
        # step's workspace, typically) is always usable; only new device
        # memory is held to the budget (which costs a driver query).
        if size > _workspace_limit(device):
            return None
    try:
        return torch.empty(size, dtype=torch.uint8, device=device)
    except torch.cuda.OutOfMemoryError:
        return None


def _bwd(q, k, v, o, lse, do, causal, window, scale, stage=None, out=None, rows=None, workspace=None):
    """Backward launches. `stage` (0 dQ+delta, 1 dK, 2 dV) runs one kernel only,
    into the buffers of `out` = (dq, dk, dv, delta) (profiling / benchmarks);
    with `rows` = (begin, end) only those rows (query rows for stage 0, key rows
    for stages 1 and 2).

    A full backward (no stage, no rows) takes the materialised
    path (gqafa_bwd_ws: the dQ kernel stores P and dS, one kernel makes dK and
    dV from them) with a workspace from the caching allocator, or `workspace`
    when given; when the whole workspace does not fit (memory or
    the budget of _workspace_limit) it runs over groups of KV heads, and without
    room for one KV head's share it runs the recomputing gqafa_bwd. With a
    `workspace` tensor, `stage` 0 / 1 selects that path's kernels instead."""
    lib = _lib.load()
    b, h_q, n, d = q.shape
    h_kv = k.shape[1]
    ws = workspace
    chunks = None
    if ws is None and stage is None and rows is None:
        size = bwd_workspace_size(b, h_q, h_kv, n, d, causal, window)
        ws = _alloc_workspace(size, q.device)
        if ws is None and size > 0:
            chunks, ws = _workspace_chunks(size, b, h_kv, q.device)
    if out is None and stage is None and rows is None and chunks is None:
        # the hot path: one torch operator call (torch_ops.cpp) over the C ABI;
        # gqafa_bwd_ws with a workspace, the recomputing gqafa_bwd without
        return _lib.ops().bwd(q, k, v, o, lse, do, bool(causal), int(window), float(scale), ws)
    q, k, v, o = _abi_ready(q), _abi_ready(k), _abi_ready(v), _abi_ready(o)
    do = _abi_ready(do)
    if out is None:
        dq = _abi_ready(torch.empty_like(q))
        dk = _abi_ready(torch.empty_like(k))
        dv = _abi_ready(torch.empty_like(v))
        delta = torch.empty((b, h_q, n), dtype=torch.float32, device=q.device)
    else:
        dq, dk, dv, delta = out
    # the C ABI reads LSE and delta as contiguous [B, H_Q, N] fp32 arrays
    if not lse.is_contiguous():
        lse = lse.contiguous()
    if not delta.is_contiguous():
        raise ValueError("delta must be a contiguous (B, H_Q, N) float32 tensor")
    if ws is not None:
        tail = (ws.data_ptr(), ws.numel() * ws.element_size())
        if stage is None:
            fn = lambda *a: lib.gqafa_bwd_ws(*a, *tail)  # noqa: E731
        else:
            fn = lambda *a: lib.gqafa_bwd_ws_stage(int(stage), *a, *tail)  # noqa: E731
    elif rows is not None:
        fn = lambda *a: lib.gqafa_bwd_stage_rows(int(stage), *a, int(rows[0]), int(rows[1]))  # noqa: E731
    else:
        fn = lib.gqafa_bwd if stage is None else (lambda *a: lib.gqafa_bwd_stage(int(stage), *a))
    with _DeviceScope(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if chunks is None:
            _lib.check(fn(*_bwd_args(q, k, v, o, do, lse, dq, dk, dv, delta, causal, window, scale, stream)))
        else:
            # the materialised backward over groups of `chunks` KV heads of one
            # batch element (units are independent; every slice is a view)
            g = h_q // h_kv
            for bi in range(b):
                for h0 in range(0, h_kv, chunks):
                    h1 = min(h_kv, h0 + chunks)
                    sq, sk, sb = slice(h0 * g, h1 * g), slice(h0, h1), slice(bi, bi + 1)
                    _lib.check(fn(*_bwd_args(
                        q[sb, sq], k[sb, sk], v[sb, sk], o[sb, sq], do[sb, sq], lse[sb, sq],
                        dq[sb, sq], dk[sb, sk], dv[sb, sk], delta[sb, sq], causal, window, scale, stream)))
    return dq, dk, dv


def _workspace_chunks(size, b, h_kv, device):
    """(KV heads per chunk, workspace) for a materialised backward split over
    groups of KV heads when the whole workspace does not fit; (None, None) if
    one KV head's share does not fit either (the caller then recomputes). The
    workspace is linear in B * H_Q, so one KV head of one batch element needs
    size / (B * H_KV)."""
    if _workspace_limit() == 0:
        return None, None
    per_head = size // (b * h_kv)
    hc = h_kv if b > 1 else h_kv // 2
    while hc >= 1:
        ws = _alloc_workspace(per_head * hc, device)
        if ws is not None:
            return hc, ws
        hc //= 2
    return None, None


def _bwd_args(q, k, v, o, do, lse, dq, dk, dv, delta, causal, window, scale, stream):
    """The gqafa_bwd argument list (without the workspace) for these tensors;
    lse and delta must be contiguous [B, H_Q, N]."""
    b, h_q, n, d = q.shape
    return (
        q.data_ptr(), _lib.strides_arg(q.stride()),
        k.data_ptr(), _lib.strides_arg(k.stride()),
        v.data_ptr(), _lib.strides_arg(v.stride()),
        o.data_ptr(), _lib.strides_arg(o.stride()),
        do.data_ptr(), _lib.strides_arg(do.stride()),
        lse.data_ptr(),
        dq.data_ptr(), _lib.strides_arg(dq.stride()),
        dk.data_ptr(), _lib.strides_arg(dk.stride()),
        dv.data_ptr(), _lib.strides_arg(dv.stride()),
        delta.data_ptr(),
        b, h_q, k.shape[1], n, d, float(scale), 1 if causal else 0, int(window),
        _DTYPES[q.dtype], stream,
    )


# --------------------------------------------------------------------------
# Public API
# --------------------------------------------------------------------------

def attention_flash_gqa(q, k, v, causal=False, slide_size=0,
                        BLOCK_Q=None, BLOCK_KV=None,
                        BLOCK_D=None, num_warps=None, num_stages=None):
    """Inference forward (no LSE, no autograd). Tile arguments are ignored.

    q: (B, H_Q, N, D); k, v: (B, H_KV, N_k, D). Returns O shaped and typed like q.

    N_k may differ from N (a KV cache, e.g. decoding): with ``causal`` the
    queries are the last N of the N_k positions (N_k >= N), and a sliding
    window counts back from each query's position; without ``causal`` every
    query sees all N_k keys. (The reference reads keys up to N only,
    attention.py:552-553.)
    """
    _check_inputs(q, k, v, kv_cache=True, causal=causal)
    window = _normalize_window(causal, slide_size, k.shape[2])
    o, _ = _fwd(q, k, v, causal, window, 1.0 / math.sqrt(q.shape[3]), want_lse=False)
    return o


class FlashAttnGQAFunction(torch.autograd.Function):
    """Autograd wrapper: forward saves (q, k, v, o, lse); backward runs the dQ
    (+ delta) kernel and the packed-GQA dK and dV kernels.

    ``apply(q, k, v, causal, slide_size[, softmax_scale])``; backward returns
    ``(dq, dk, dv, None, None, None)`` with gradients in the input dtype.
    """

    @staticmethod
    def forward(ctx, q, k, v, causal, slide_size, softmax_scale=None):
        _check_inputs(q, k, v)
        n, d = q.shape[2], q.shape[3]
        window = _normalize_window(causal, slide_size, n)
        scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
        o, lse = _fwd(q, k, v, causal, window, scale, want_lse=True)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = bool(causal)
        ctx.window = window
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _bwd(q, k, v, o, lse, do, ctx.causal, ctx.window, ctx.scale)
        return dq, dk, dv, None, None, None


def flash_attn_gqa_train(q, k, v, causal=False, slide_size=0):
    """Training forward with backward support (autograd)."""
    return FlashAttnGQAFunction.apply(q, k, v, causal, slide_size)


def flash_attn_gqa_forward_with_lse(q, k, v, causal=False, slide_size=0, softmax_scale=None):
    """Forward returning (O, LSE); LSE is fp32 (B, H_Q, N), natural log, scaled.

    Not in the reference's public API; used by tests and the multi-GPU path.
    Accepts a KV cache longer than the queries as attention_flash_gqa does.
    """
    _check_inputs(q, k, v, kv_cache=True, causal=causal)
    window = _normalize_window(causal, slide_size, k.shape[2])
    scale = (1.0 / math.sqrt(q.shape[3])) if softmax_scale is None else float(softmax_scale)
    return _fwd(q, k, v, causal, window, scale, want_lse=True)


def flash_attn_gqa_backward(q, k, v, o, lse, do, causal=False, slide_size=0, softmax_scale=None):
    """Explicit backward: returns (dq, dk, dv). Not in the reference's public API."""
    _check_inputs(q, k, v)
    window = _normalize_window(causal, slide_size, q.shape[2])
    scale = (1.0 / math.sqrt(q.shape[3])) if softmax_scale is None else float(softmax_scale)
    return _bwd(q, k, v, o, lse, do, causal, window, scale)
