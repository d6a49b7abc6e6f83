"""TEST INFRASTRUCTURE ONLY. CPU checker for blackflash_b200.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module. The product path (blackflash_b200) never imports it.

Contents:
  attn_exact   the C restatement of the reference's fp32 math attention
               (reference tests/test_blackflash.py:16-19, profile/gen_ref.py:80-84),
               accumulated in double. Returns O, lse and the row max in fp32.
  attn_fa2     the C restatement of the reference kernel's tiled online-softmax
               algorithm (kernel/flash_attn_mma.cu:228-464). Returns a bf16-rounded O.
  attn_bwd     gradients dQ, dK, dV of the same forward for an upstream dO, in double
               (attn_bwd_oracle.c; the reference has no backward, so it is pinned
               against torch autograd of the fp32 forward instead).
  scores       S = QK^T * scale and P = softmax(S) of one slice, which is what
               gen_ref.py saves as s_ref.bin / p_ref.bin (:80-84).
  attn_numpy   a float64 numpy statement of the same formula, used to cross-check
               the C code on tiny cases.
  torch_math   the reference's CPU formula literally, in torch fp32
               (tests/test_blackflash.py:16-19). The CPU baseline times it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    srcs = [os.path.join(HERE, f) for f in ("attn_oracle.c", "attn_bwd_oracle.c")]
    if not os.path.exists(LIB) or any(os.path.getmtime(LIB) < os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True, capture_output=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        vp, ll, i, f = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_float
        lib.oracle_attn_exact.argtypes = [vp, vp, vp, vp, vp, vp, ll, i, i, i, f, i]
        lib.oracle_attn_exact_causal.argtypes = [vp, vp, vp, vp, vp, vp, ll, i, i, i, f, i, i]
        lib.oracle_attn_exact_causal.restype = i
        lib.oracle_attn_fa2.argtypes = [vp, vp, vp, vp, vp, vp, ll, i, i, f, i]
        lib.oracle_scores.argtypes = [vp, vp, vp, vp, i, i, f]
        lib.oracle_attn_bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, ll, i, i, f, i]
        lib.oracle_attn_bwd.restype = i
        for fn in (lib.oracle_attn_exact, lib.oracle_attn_fa2, lib.oracle_scores):
            fn.restype = i
        _lib = lib
    return _lib


def as_bf16_bits(x) -> np.ndarray:
    """torch bf16 tensor or uint16 array -> contiguous uint16 numpy array of bf16 bits."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            assert x.dtype == torch.bfloat16
            return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    except ImportError:  # pragma: no cover
        pass
    a = np.ascontiguousarray(x)
    assert a.dtype == np.uint16
    return a


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def attn_exact(q, k, v, scale: float, nthreads: int | None = None, causal: bool = False):
    """q: [..., Nq, d], k/v: [..., Nkv, d] bf16. Returns (O, lse, rowmax) fp32 numpy.
    causal=True masks key j for query i when j > i."""
    qb, kb, vb = as_bf16_bits(q), as_bf16_bits(k), as_bf16_bits(v)
    *lead, nq, d = qb.shape
    nkv = kb.shape[-2]
    bh = int(np.prod(lead)) if lead else 1
    o = np.empty(qb.shape, dtype=np.float32)
    lse = np.empty((*lead, nq), dtype=np.float32)
    mx = np.empty((*lead, nq), dtype=np.float32)
    _load().oracle_attn_exact_causal(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(o), _ptr(lse), _ptr(mx), bh, nq, nkv, d,
                                     float(scale), 1 if causal else 0, nthreads or os.cpu_count() or 1)
    return o, lse, mx


def attn_fa2(q, k, v, scale: float, nthreads: int | None = None):
    """The reference kernel's algorithm (64x64 tiles, bf16 P). Returns (O bf16-rounded fp32, lse, rowmax)."""
    qb, kb, vb = as_bf16_bits(q), as_bf16_bits(k), as_bf16_bits(v)
    *lead, n, d = qb.shape
    bh = int(np.prod(lead)) if lead else 1
    o = np.empty(qb.shape, dtype=np.float32)
    lse = np.empty((*lead, n), dtype=np.float32)
    mx = np.empty((*lead, n), dtype=np.float32)
    _load().oracle_attn_fa2(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(o), _ptr(lse), _ptr(mx), bh, n, d, float(scale),
                            nthreads or os.cpu_count() or 1)
    return o, lse, mx


def attn_bwd(q, k, v, dout, scale: float, nthreads: int | None = None):
    """Gradients of O = softmax(scale Q K^T) V for upstream dO, all bf16 [..., N, d].
    Returns (dQ, dK, dV) fp32 numpy, computed in double (attn_bwd_oracle.c)."""
    qb, kb, vb, gb = as_bf16_bits(q), as_bf16_bits(k), as_bf16_bits(v), as_bf16_bits(dout)
    *lead, n, d = qb.shape
    bh = int(np.prod(lead)) if lead else 1
    dq, dk, dv = (np.empty(qb.shape, dtype=np.float32) for _ in range(3))
    _load().oracle_attn_bwd(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(gb), _ptr(dq), _ptr(dk), _ptr(dv), bh, n, d,
                            float(scale), nthreads or os.cpu_count() or 1)
    return dq, dk, dv


def scores(q_slice, k_slice, scale: float):
    """One slice [N, d] each. Returns (S, P) fp32 [N, N]."""
    qb, kb = as_bf16_bits(q_slice), as_bf16_bits(k_slice)
    n, d = qb.shape
    s = np.empty((n, n), dtype=np.float32)
    p = np.empty((n, n), dtype=np.float32)
    _load().oracle_scores(_ptr(qb), _ptr(kb), _ptr(s), _ptr(p), n, d, float(scale))
    return s, p


def attn_numpy(q, k, v, scale: float, causal: bool = False):
    """float64 numpy math attention on bf16 inputs; returns (O, lse) float64."""
    qf = bf16_bits_to_f32(as_bf16_bits(q)).astype(np.float64)
    kf = bf16_bits_to_f32(as_bf16_bits(k)).astype(np.float64)
    vf = bf16_bits_to_f32(as_bf16_bits(v)).astype(np.float64)
    s = np.einsum("...id,...jd->...ij", qf, kf) * scale
    if causal:
        nq, nk = s.shape[-2], s.shape[-1]
        s = np.where(np.arange(nk)[None, :] <= np.arange(nq)[:, None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    den = e.sum(axis=-1, keepdims=True)
    o = np.einsum("...ij,...jd->...id", e / den, vf)
    return o, (m + np.log(den))[..., 0]


def torch_math(Q, K, V, scale: float):
    """Reference CPU formula (tests/test_blackflash.py:16-19) in torch fp32: returns fp32 O."""
    import torch
    S = torch.matmul(Q.float(), K.float().transpose(-1, -2)) * scale
    P = torch.softmax(S, dim=-1)
    return torch.matmul(P, V.float())
