"""Torch-facing operators over the C ABI.

`forward` mirrors the reference's torch extension function
`blackflash_cuda.forward` (binding/blackflash_ops.cu:18-55): same argument
order and meaning, same checks (CUDA, bf16, contiguous, d == 64; d == 128 is accepted as an extension), the same
RuntimeError on a failed check, and a fresh bf16 O as the result. What differs:
  * it launches on Q's device (the reference has no device guard and uses
    whatever device is current);
  * it does not allocate and fill the unused l/m buffers on every call;
  * K and V must have Q's shape (the reference reads them with Q's sizes
    without checking).
"""
from __future__ import annotations

import math

import torch

from . import _lib


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_qkv(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> None:
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        _require(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
        _require(t.is_cuda and t.dtype == torch.bfloat16, f"{name} must be a CUDA bfloat16 tensor")
        _require(t.is_contiguous(), f"{name} must be contiguous")
        _require(t.dim() == 4, f"{name} must be [B, H, N, d]")
    _require(K.shape == Q.shape and V.shape == Q.shape, "Q, K and V must have the same shape")
    _require(K.device == Q.device and V.device == Q.device, "Q, K and V must be on the same device")
    _require(Q.size(3) in (64, 128), "BlackFlash supports d=64 and d=128")


def _stream_handle(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float) -> torch.Tensor:
    """O = softmax(scale * Q K^T) V; bf16 [B, H, N, d] in and out, d = 64 or 128."""
    return forward_lse(Q, K, V, scale, want_stats=False)[0]


def forward_lse(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float, want_stats: bool = True,
                causal: bool = False):
    """Like `forward`, and also returns (lse, row_max), each fp32 [B, H, N].

    causal=True applies a causal mask (query i sees keys j <= i); the reference
    has no causal kernel, so this is an extension (its default is off).

    lse[b,h,i] = log sum_j exp(scale * S_ij) and row_max[b,h,i] = max_j scale * S_ij:
    the two quantities the reference's l/m slots were declared for
    (include/flash_attn.cuh:27-28).
    """
    _check_qkv(Q, K, V)
    B, H, N, d = Q.shape
    O = torch.empty_like(Q)
    lse = m = None
    if want_stats:
        lse = torch.empty((B, H, N), dtype=torch.float32, device=Q.device)
        m = torch.empty((B, H, N), dtype=torch.float32, device=Q.device)
    if Q.numel() == 0:
        return O, lse, m
    lib = _lib.load()
    fn = lib.blackflash_fwd_causal if causal else lib.blackflash_fwd
    with torch.cuda.device(Q.device):
        rc = fn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                lse.data_ptr() if lse is not None else None,
                m.data_ptr() if m is not None else None,
                B, H, N, d, float(scale), _stream_handle(Q.device))
    _lib.check(rc, "blackflash_fwd_causal" if causal else "blackflash_fwd")
    return O, lse, m


def blackflash(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float | None = None,
               causal: bool = False) -> torch.Tensor:
    """Attention forward. Mirrors the reference's Python API (blackflash/__init__.py:5-18):
    Q, K, V are [B, H, N, d] bf16 CUDA tensors with d == 64 (the reference's only size) or 128; scale defaults to 1/sqrt(d).
    `causal` (default False, the reference's only mode) is an extension."""
    if scale is None:
        scale = 1.0 / math.sqrt(Q.size(-1))
    if causal:
        return forward_lse(Q, K, V, scale, want_stats=False, causal=True)[0]
    return forward(Q, K, V, scale)


def attention_partial(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float):
    """One ring step: Q [S, Nq, 64] against K/V [S, Nkv, 64] (S = flattened slices).

    Returns (O_f32 [S, Nq, 64] normalised over this KV block, lse [S, Nq])."""
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.dim() == 3,
                 f"{name} must be a contiguous CUDA bf16 [slices, rows, 64] tensor")
    _require(Q.size(0) == K.size(0) == V.size(0) and K.shape == V.shape and Q.size(2) == 64 and K.size(2) == 64,
             "partial attention needs Q [S,Nq,64] and K,V [S,Nkv,64]")
    S, Nq, _ = Q.shape
    Nkv = K.size(1)
    O = torch.empty((S, Nq, 64), dtype=torch.float32, device=Q.device)
    lse = torch.empty((S, Nq), dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    with torch.cuda.device(Q.device):
        rc = lib.blackflash_fwd_partial(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr(),
                                        S, Nq, Nkv, 64, float(scale), _stream_handle(Q.device))
    _lib.check(rc, "blackflash_fwd_partial")
    return O, lse


def attention_partial_blocks(Q: torch.Tensor, Kg: torch.Tensor, Vg: torch.Tensor, scale: float, skip: int = -1):
    """Q [S, Nq, 64] against the gathered blocks Kg, Vg [G, S, n, 64] with block `skip`
    left out (-1: all blocks). n must be a multiple of 128.

    Returns (O_f32 [S, Nq, 64], lse [S, Nq]) over the concatenated used blocks."""
    for name, t in (("Q", Q), ("Kg", Kg), ("Vg", Vg)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous(), f"{name} must be a contiguous CUDA bf16 tensor")
    _require(Q.dim() == 3 and Kg.dim() == 4 and Kg.shape == Vg.shape and Q.size(2) == 64 and Kg.size(3) == 64
             and Kg.size(1) == Q.size(0), "partial_blocks needs Q [S,Nq,64] and Kg, Vg [G,S,n,64]")
    S, Nq, _ = Q.shape
    G, _, n, _ = Kg.shape
    O = torch.empty((S, Nq, 64), dtype=torch.float32, device=Q.device)
    lse = torch.empty((S, Nq), dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    with torch.cuda.device(Q.device):
        rc = lib.blackflash_fwd_partial_blocks(Q.data_ptr(), Kg.data_ptr(), Vg.data_ptr(), O.data_ptr(), lse.data_ptr(),
                                               S, Nq, G, n, int(skip), 64, float(scale), _stream_handle(Q.device))
    _lib.check(rc, "blackflash_fwd_partial_blocks")
    return O, lse


def attention_backward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, O: torch.Tensor, dO: torch.Tensor,
                       lse: torch.Tensor, scale: float):
    """Gradients (dQ, dK, dV) of O = softmax(scale Q K^T) V for upstream dO.

    Q, K, V, O, dO: [B, H, N, 64] bf16 CUDA; lse: [B, H, N] fp32 from `forward_lse`.
    Non-causal, d = 64. The fp32 workspace (a dQ accumulator and two row vectors)
    is allocated here from torch's caching allocator."""
    _check_qkv(Q, K, V)
    for name, t in (("O", O), ("dO", dO)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.shape == Q.shape,
                 f"{name} must be a contiguous CUDA bf16 tensor of Q's shape")
    _require(lse.is_cuda and lse.dtype == torch.float32 and lse.is_contiguous() and lse.shape == Q.shape[:3],
             "lse must be a contiguous CUDA fp32 [B, H, N] tensor")
    _require(Q.size(3) == 64, "the backward supports d=64")
    B, H, N, d = Q.shape
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(Q), torch.empty_like(Q)
    if Q.numel() == 0:
        return dQ, dK, dV
    lib = _lib.load()
    nbytes = lib.blackflash_bwd_workspace_bytes(B, H, N, d)
    ws = torch.empty(nbytes // 4, dtype=torch.float32, device=Q.device)
    with torch.cuda.device(Q.device):
        rc = lib.blackflash_bwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), dO.data_ptr(), lse.data_ptr(),
                                dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), ws.data_ptr(), nbytes, B, H, N, d,
                                float(scale), _stream_handle(Q.device))
    _lib.check(rc, "blackflash_bwd")
    return dQ, dK, dV


class _BlackFlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, scale):
        O, lse, _ = forward_lse(Q, K, V, scale, want_stats=True)
        ctx.save_for_backward(Q, K, V, O, lse)
        ctx.scale = scale
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, lse = ctx.saved_tensors
        dQ, dK, dV = attention_backward(Q, K, V, O, dO.contiguous(), lse, ctx.scale)
        return dQ, dK, dV, None


def blackflash_with_grad(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """`blackflash` as a differentiable op (forward and backward on the sm_100a kernels)."""
    if scale is None:
        scale = 1.0 / math.sqrt(Q.size(-1))
    return _BlackFlashFn.apply(Q, K, V, float(scale))


def lse_merge_(O_acc: torch.Tensor, lse_acc: torch.Tensor, O_part: torch.Tensor, lse_part: torch.Tensor) -> None:
    """In-place log-sum-exp merge of a partial result into the running one (fp32)."""
    for t in (O_acc, lse_acc, O_part, lse_part):
        _require(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous(), "merge operands must be contiguous CUDA fp32")
    rows = lse_acc.numel()
    _require(O_acc.numel() == rows * 64 and O_part.numel() == rows * 64 and lse_part.numel() == rows,
             "merge operands disagree in size")
    lib = _lib.load()
    with torch.cuda.device(O_acc.device):
        rc = lib.blackflash_lse_merge(O_acc.data_ptr(), lse_acc.data_ptr(), O_part.data_ptr(), lse_part.data_ptr(),
                                      rows, 64, _stream_handle(O_acc.device))
    _lib.check(rc, "blackflash_lse_merge")


def to_bf16(src: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 through the library's cast kernel."""
    _require(src.is_cuda and src.dtype == torch.float32 and src.is_contiguous(), "src must be contiguous CUDA fp32")
    dst = torch.empty(src.shape, dtype=torch.bfloat16, device=src.device)
    if src.numel():
        lib = _lib.load()
        with torch.cuda.device(src.device):
            rc = lib.blackflash_f32_to_bf16(src.data_ptr(), dst.data_ptr(), src.numel(), _stream_handle(src.device))
        _lib.check(rc, "blackflash_f32_to_bf16")
    return dst


def wait_status(reset: bool = True) -> int:
    """Device-side wait-timeout status of the current device (0 = none). Synchronous."""
    import ctypes
    out = ctypes.c_uint(0)
    _lib.check(_lib.load().blackflash_status(1 if reset else 0, ctypes.byref(out)), "blackflash_status")
    return int(out.value)


def blackflash_host(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float | None = None,
                    causal: bool = False, device: torch.device | int | str = 0, chunks: int = 8,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention forward for Q, K, V held in (preferably pinned) host memory.

    The (b, h) slices are processed in `chunks` groups on three CUDA streams, so the
    host->device copy of group i+1, the kernel on group i and the device->host copy of
    group i-1 run at the same time; the transfer, not the kernel, bounds the call.
    Returns O in host memory (pinned, or `out` if given). Synchronous: O is ready when
    the call returns.
    """
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        _require(not t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.dim() == 4,
                 f"{name} must be a contiguous host bf16 [B, H, N, d] tensor")
    _require(K.shape == Q.shape and V.shape == Q.shape, "Q, K and V must have the same shape")
    _require(Q.size(3) in (64, 128), "BlackFlash supports d=64 and d=128")
    B, H, N, d = Q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    if out is None:
        out = torch.empty(Q.shape, dtype=Q.dtype, pin_memory=True)
    _require(out.shape == Q.shape and out.dtype == Q.dtype and not out.is_cuda and out.is_contiguous(),
             "out must be a contiguous host bf16 tensor of Q's shape")
    S = B * H
    if S == 0 or N == 0:
        return out
    qs, ks, vs, os_ = (t.view(S, 1, N, d) for t in (Q, K, V, out))
    chunks = max(1, min(chunks, S))
    lib = _lib.load()
    bounds = [(S * i // chunks, S * (i + 1) // chunks) for i in range(chunks)]
    with torch.cuda.device(dev):
        dq, dk, dv = (torch.empty((S, 1, N, d), dtype=Q.dtype, device=dev) for _ in range(3))
        do = torch.empty((S, 1, N, d), dtype=Q.dtype, device=dev)
        h2d, comp, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        caller = torch.cuda.current_stream(dev)
        for st in (h2d, comp, d2h):
            st.wait_stream(caller)
        for a, b in bounds:
            if b == a:
                continue
            with torch.cuda.stream(h2d):
                dq[a:b].copy_(qs[a:b], non_blocking=True)
                dk[a:b].copy_(ks[a:b], non_blocking=True)
                dv[a:b].copy_(vs[a:b], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(ev_in)
                fn = lib.blackflash_fwd_causal if causal else lib.blackflash_fwd
                _lib.check(fn(dq[a:b].data_ptr(), dk[a:b].data_ptr(), dv[a:b].data_ptr(), do[a:b].data_ptr(),
                              None, None, b - a, 1, N, d, float(scale), comp.cuda_stream), "blackflash_host")
                ev_out = torch.cuda.Event()
                ev_out.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_out)
                os_[a:b].copy_(do[a:b], non_blocking=True)
        for st in (h2d, comp, d2h):
            caller.wait_stream(st)
        d2h.synchronize()
    return out
