"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU oracle (attn_oracle.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker.  It restates attention.metal:19-299 on the CPU (see
the header of attn_oracle.cpp); PARITY UNPINNED: the reference ships no golden
vectors and cannot run off Apple hardware.

All arrays are numpy: bf16 tensors are uint16 bit patterns in the reference
layout ([B, T, N] activations, [B, T, NH] row statistics).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libattn_oracle.so"

EXACT, FAITHFUL, FP64 = 0, 1, 2

_lib = None


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            import sys
            sys.path.insert(0, str(HERE.parent))
            from metalllm_b200.build import build_oracle
            build_oracle()
        lib = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        U = ctypes.c_uint32
        I = ctypes.c_int
        lib.oracle_compute_qkv.argtypes = [P, P, P, P, P, P, P, U, U, U, I, P, P, P]
        lib.oracle_flash_forward.argtypes = [P, P, P, P, P, U, U, U, U, U, U, U, I, I, P]
        lib.oracle_compute_d.argtypes = [P, P, P, U, U, U, U, U, U, U, I, I, P]
        lib.oracle_flash_backward.argtypes = [P, P, P, P, P, P, P, P, P, U, U, U, U, U, U, U, I, I, P, P]
        lib.oracle_fp64_loss.argtypes = [P, P, P, P, U, U]
        lib.oracle_fp64_loss.restype = ctypes.c_double
        L = ctypes.c_int64
        lib.oracle_proj_forward.argtypes = [P, P, P, U, U, P, L, I, P]
        lib.oracle_proj_backward_dx.argtypes = [P, P, P, U, U, P, L, I, P]
        lib.oracle_proj_backward_dw.argtypes = [P, P, P, U, U, P, L, I, P]
        lib.oracle_grad_dx.argtypes = [P, P, P, P, P, P, P, U, U, P, L, I]
        lib.oracle_grad_dw.argtypes = [P, P, P, P, P, P, P, U, U, P, L, I, P, P]
        for n in ("oracle_compute_qkv", "oracle_flash_forward", "oracle_compute_d",
                  "oracle_flash_backward", "oracle_proj_forward", "oracle_proj_backward_dx",
                  "oracle_proj_backward_dw", "oracle_grad_dx", "oracle_grad_dw"):
            getattr(lib, n).restype = ctypes.c_int
        _lib = lib
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def default_threads() -> int:
    return os.cpu_count() or 1


def _shape(q, NH):
    B, T, N = q.shape
    return B, T, N, N // NH


def compute_qkv(X, qw, kw, vw, nthreads=0, want_f32=False):
    rows, N = X.shape[0] * X.shape[1], X.shape[2]
    B, M = X.shape[0], X.shape[1]
    q = np.empty_like(X); k = np.empty_like(X); v = np.empty_like(X)
    f = [np.empty(X.shape, np.float32) for _ in range(3)] if want_f32 else [None] * 3
    rc = load().oracle_compute_qkv(_p(X), _p(q), _p(k), _p(v), _p(qw), _p(kw), _p(vw), M, N, B,
                                   nthreads, _p(f[0]), _p(f[1]), _p(f[2]))
    assert rc == 0
    return (q, k, v, *f) if want_f32 else (q, k, v)


def flash_forward(q, k, v, NH, mode=EXACT, shard=None, nthreads=0, out=None, lse=None,
                  want_f32=False):
    B, T, N, D = _shape(q, NH)
    out = np.zeros_like(q) if out is None else out
    lse = np.zeros((B, T, NH), np.float32) if lse is None else lse
    o32 = np.zeros(q.shape, np.float32) if want_f32 else None
    b0, b1 = shard if shard is not None else (0, B * NH)
    rc = load().oracle_flash_forward(_p(q), _p(k), _p(v), _p(out), _p(lse), T, N, D, NH, B, b0, b1,
                                     mode, nthreads, _p(o32))
    assert rc == 0, "oracle_flash_forward rejected its arguments"
    return (out, lse, o32) if want_f32 else (out, lse)


def compute_d(dO, O, NH, mode=EXACT, shard=None, nthreads=0, want_f32=False):
    B, T, N, D = _shape(dO, NH)
    Dv = np.zeros((B, T, NH), np.uint16)
    d32 = np.zeros((B, T, NH), np.float32) if want_f32 else None
    b0, b1 = shard if shard is not None else (0, B * NH)
    rc = load().oracle_compute_d(_p(dO), _p(O), _p(Dv), T, N, D, NH, B, b0, b1, mode, nthreads,
                                 _p(d32))
    assert rc == 0
    return (Dv, d32) if want_f32 else Dv


def flash_backward(dO, Dv, lse, q, k, v, NH, mode=EXACT, shard=None, nthreads=0, want_f32=False):
    B, T, N, D = _shape(q, NH)
    dQ = np.zeros(q.shape, np.float32)
    dK = np.zeros_like(q)
    dV = np.zeros_like(q)
    dk32 = np.zeros(q.shape, np.float32) if want_f32 else None
    dv32 = np.zeros(q.shape, np.float32) if want_f32 else None
    b0, b1 = shard if shard is not None else (0, B * NH)
    rc = load().oracle_flash_backward(_p(dO), _p(Dv), _p(lse), _p(q), _p(k), _p(v), _p(dQ), _p(dK),
                                      _p(dV), T, N, D, NH, B, b0, b1, mode, nthreads, _p(dk32),
                                      _p(dv32))
    assert rc == 0, "oracle_flash_backward rejected its arguments"
    return (dQ, dK, dV, dk32, dv32) if want_f32 else (dQ, dK, dV)


def fp64_loss(q, k, v, dO):
    """sum(dO * attention(q, k, v)) in fp64 for one head; q..dO are fp64 [T, D]."""
    T, D = q.shape
    arrs = [np.ascontiguousarray(a, dtype=np.float64) for a in (q, k, v, dO)]
    return load().oracle_fp64_loss(*[_p(a) for a in arrs], T, D)


def bf16_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def compare(got, want, max_abs=2e-2, rel_l2=1e-2):
    """Max-abs and relative-L2 errors of got vs want (float arrays); returns
    (ok, max_abs_err, rel_l2_err)."""
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    err = np.abs(g - w)
    mae = float(err.max()) if err.size else 0.0
    denom = float(np.linalg.norm(w))
    rl2 = float(np.linalg.norm(g - w) / denom) if denom > 0 else float(np.linalg.norm(g - w))
    ok = bool(np.isfinite(g).all()) and mae <= max_abs and rl2 <= rel_l2
    return ok, mae, rl2


# ------------------------------------------------------------------ GEMMs
# attention.metal:301-455.  Activations are [rows, N] (any leading shape is
# flattened), weights [N, N] bf16 bits; dQ and the fp32 outputs are float32.
# `rows` (optional) restricts the computed output rows; the others are NaN.

def _sel(rows):
    if rows is None:
        return None, 0
    r = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    return r, len(r)


def _flat(a):
    return np.ascontiguousarray(a).reshape(-1, a.shape[-1])


def proj_forward(attn, w, rows=None, nthreads=0):
    """out = attn . w (attention.metal:395-416); returns (bf16 bits, fp32)."""
    a = _flat(attn); R, N = a.shape
    out = np.full(a.shape, 0x7FC0, np.uint16); o32 = np.full(a.shape, np.nan, np.float32)
    sel, ns = _sel(rows)
    assert load().oracle_proj_forward(_p(a), _p(w), _p(out), R, N, _p(sel), ns, nthreads, _p(o32)) == 0
    return out, o32


def proj_backward_dx(dz, w, rows=None, nthreads=0):
    """dAttn = dz . w^T (attention.metal:432-455); returns (bf16 bits, fp32)."""
    a = _flat(dz); R, N = a.shape
    out = np.full(a.shape, 0x7FC0, np.uint16); o32 = np.full(a.shape, np.nan, np.float32)
    sel, ns = _sel(rows)
    assert load().oracle_proj_backward_dx(_p(a), _p(w), _p(out), R, N, _p(sel), ns, nthreads, _p(o32)) == 0
    return out, o32


def proj_backward_dw(attn, dz, rows=None, nthreads=0):
    """dW = attn^T . dz (attention.metal:418-430); returns (bf16 bits, fp32) [N, N]."""
    a = _flat(attn); g = _flat(dz); R, N = a.shape
    out = np.full((N, N), 0x7FC0, np.uint16); o32 = np.full((N, N), np.nan, np.float32)
    sel, ns = _sel(rows)
    assert load().oracle_proj_backward_dw(_p(a), _p(g), _p(out), R, N, _p(sel), ns, nthreads, _p(o32)) == 0
    return out, o32


def grad_dx(qw, kw, vw, dq, dk, dv, rows=None, nthreads=0):
    """dX = dQ.Wq^T + dK.Wk^T + dV.Wv^T, fp32 (attention.metal:301-342)."""
    q32 = np.ascontiguousarray(dq, dtype=np.float32).reshape(-1, dq.shape[-1])
    k = _flat(dk); v = _flat(dv); R, N = k.shape
    dx = np.full((R, N), np.nan, np.float32)
    sel, ns = _sel(rows)
    assert load().oracle_grad_dx(_p(dx), _p(qw), _p(kw), _p(vw), _p(q32), _p(k), _p(v), R, N,
                                 _p(sel), ns, nthreads) == 0
    return dx


def grad_dw(x, dq, dk, dv, rows=None, nthreads=0):
    """dQw = X^T.dQ (fp32), dKw = X^T.dK, dVw = X^T.dV (attention.metal:344-393).
    Returns dQw, dKw bits, dVw bits, dKw fp32, dVw fp32 ([N, N] each)."""
    xx = _flat(x); R, N = xx.shape
    q32 = np.ascontiguousarray(dq, dtype=np.float32).reshape(-1, N)
    k = _flat(dk); v = _flat(dv)
    dqw = np.full((N, N), np.nan, np.float32)
    dkw = np.full((N, N), 0x7FC0, np.uint16); dvw = np.full((N, N), 0x7FC0, np.uint16)
    k32 = np.full((N, N), np.nan, np.float32); v32 = np.full((N, N), np.nan, np.float32)
    sel, ns = _sel(rows)
    assert load().oracle_grad_dw(_p(xx), _p(q32), _p(k), _p(v), _p(dqw), _p(dkw), _p(dvw), R, N,
                                 _p(sel), ns, nthreads, _p(k32), _p(v32)) == 0
    return dqw, dkw, dvw, k32, v32
