"""Operator interface of the attention hot path on torch CUDA tensors.

The four functions mirror the reference's four kernels (attention.metal:19-299)
with the same buffer roles, order and dtypes, as its host code binds them
(model.h:446-473 forward, model.h:639-665 backward).  Each call goes through the
C ABI of libmetalattn (include/metalattn.h); PyTorch only provides the device
memory and the stream.  Outputs may be passed in (as the reference's
preallocated buffers) or are allocated here.

Shapes (B sequences of length T = params.M, N = params.N = NH*D):
    X, q, k, v, out, dO, dK, dV : bf16 [B, T, N]
    dQ                          : fp32 [B, T, N]
    l                           : fp32 [B, T, NH]
    D                           : bf16 [B, T, NH]
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import AttentionParams, MetalAttnError  # noqa: F401  (re-exported)


def make_params(T: int, NH: int, D: int) -> AttentionParams:
    """AttentionParams{M=T, N=NH*D, D, NH} as model.h:178 fills it."""
    return AttentionParams(T, NH * D, D, NH)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _check(t: torch.Tensor, name: str, dtype: torch.dtype, shape: tuple) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path exists)")
    cur = torch.cuda.current_device()
    if t.device.index != cur:
        # the entry points launch on the current device; another device's
        # pointer would be dereferenced from there
        raise ValueError(f"{name} is on {t.device} but the current CUDA device is cuda:{cur}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape) and t.numel() != _numel(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _numel(shape: tuple) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


def _out(t: Optional[torch.Tensor], like: torch.Tensor, shape: tuple, dtype: torch.dtype,
         name: str) -> torch.Tensor:
    if t is None:
        return torch.empty(shape, dtype=dtype, device=like.device)
    _check(t, name, dtype, shape)
    return t


def computeQKV(X: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, v_w: torch.Tensor,
               p: AttentionParams, B: int, q: Optional[torch.Tensor] = None,
               k: Optional[torch.Tensor] = None, v: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None):
    """q, k, v = X Wq, X Wk, X Wv (attention.metal:19-53)."""
    act = (B, p.M, p.N)
    _check(X, "X", torch.bfloat16, act)
    for w, n in ((q_w, "q_w"), (k_w, "k_w"), (v_w, "v_w")):
        _check(w, n, torch.bfloat16, (p.N, p.N))
    q = _out(q, X, act, torch.bfloat16, "q")
    k = _out(k, X, act, torch.bfloat16, "k")
    v = _out(v, X, act, torch.bfloat16, "v")
    _lib.call("ma_computeQKV", _ptr(X), _ptr(q), _ptr(k), _ptr(v), _ptr(q_w), _ptr(k_w),
              _ptr(v_w), ctypes.byref(p), B, _stream(stream))
    return q, k, v


def projForward(attn_out: torch.Tensor, proj_w: torch.Tensor, p: AttentionParams, B: int,
                out: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None):
    """out = attn_out . proj_w (attention.metal:395-416)."""
    act = (B, p.M, p.N)
    _check(attn_out, "attn_out", torch.bfloat16, act)
    _check(proj_w, "proj_w", torch.bfloat16, (p.N, p.N))
    out = _out(out, attn_out, act, torch.bfloat16, "out")
    _lib.call("ma_projForward", _ptr(attn_out), _ptr(proj_w), _ptr(out), ctypes.byref(p), B,
              _stream(stream))
    return out


def projBackwarddW(attn_out: torch.Tensor, dZ: torch.Tensor, p: AttentionParams, B: int,
                   dProjw: Optional[torch.Tensor] = None,
                   stream: Optional[torch.cuda.Stream] = None):
    """dProjw = attn_out^T . dZ over all B*M rows (attention.metal:418-430)."""
    act = (B, p.M, p.N)
    _check(attn_out, "attn_out", torch.bfloat16, act)
    _check(dZ, "dZ", torch.bfloat16, act)
    dProjw = _out(dProjw, attn_out, (p.N, p.N), torch.bfloat16, "dProjw")
    _lib.call("ma_projBackwarddW", _ptr(attn_out), _ptr(dZ), _ptr(dProjw), ctypes.byref(p), B,
              _stream(stream))
    return dProjw


def projBackwarddX(dZ: torch.Tensor, proj_w: torch.Tensor, p: AttentionParams, B: int,
                   dAttn: Optional[torch.Tensor] = None,
                   stream: Optional[torch.cuda.Stream] = None):
    """dAttn = dZ . proj_w^T (attention.metal:432-455)."""
    act = (B, p.M, p.N)
    _check(dZ, "dZ", torch.bfloat16, act)
    _check(proj_w, "proj_w", torch.bfloat16, (p.N, p.N))
    dAttn = _out(dAttn, dZ, act, torch.bfloat16, "dAttn")
    _lib.call("ma_projBackwarddX", _ptr(dZ), _ptr(proj_w), _ptr(dAttn), ctypes.byref(p), B,
              _stream(stream))
    return dAttn


def projBackwarddXComputeD(dZ: torch.Tensor, proj_w: torch.Tensor, attn_out: torch.Tensor,
                           p: AttentionParams, B: int, dAttn: Optional[torch.Tensor] = None,
                           D: Optional[torch.Tensor] = None,
                           stream: Optional[torch.cuda.Stream] = None):
    """dAttn = dZ . proj_w^T and D = computeD(dAttn, attn_out) in one launch
    (the D sums formed in the GEMM epilogue)."""
    act = (B, p.M, p.N)
    _check(dZ, "dZ", torch.bfloat16, act)
    _check(proj_w, "proj_w", torch.bfloat16, (p.N, p.N))
    _check(attn_out, "attn_out", torch.bfloat16, act)
    dAttn = _out(dAttn, dZ, act, torch.bfloat16, "dAttn")
    D = _out(D, dZ, (B, p.M, p.NH), torch.bfloat16, "D")
    _lib.call("ma_projBackwarddXComputeD", _ptr(dZ), _ptr(proj_w), _ptr(dAttn), _ptr(attn_out), _ptr(D),
              ctypes.byref(p), B, _stream(stream))
    return dAttn, D


def computeGradDx(q_w: torch.Tensor, k_w: torch.Tensor, v_w: torch.Tensor, dQ: torch.Tensor,
                  dK: torch.Tensor, dV: torch.Tensor, p: AttentionParams, B: int,
                  dX: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None):
    """dX = dQ.Wq^T + dK.Wk^T + dV.Wv^T in fp32 (attention.metal:301-342)."""
    act = (B, p.M, p.N)
    for w, n in ((q_w, "q_w"), (k_w, "k_w"), (v_w, "v_w")):
        _check(w, n, torch.bfloat16, (p.N, p.N))
    _check(dQ, "dQ", torch.float32, act)
    _check(dK, "dK", torch.bfloat16, act)
    _check(dV, "dV", torch.bfloat16, act)
    dX = _out(dX, dK, act, torch.float32, "dX")
    _lib.call("ma_computeGradDx", _ptr(dX), _ptr(q_w), _ptr(k_w), _ptr(v_w), _ptr(dQ), _ptr(dK),
              _ptr(dV), ctypes.byref(p), B, _stream(stream))
    return dX


def computeGradDw(x: torch.Tensor, dQ: torch.Tensor, dK: torch.Tensor, dV: torch.Tensor,
                  p: AttentionParams, B: int, dQw: Optional[torch.Tensor] = None,
                  dKw: Optional[torch.Tensor] = None, dVw: Optional[torch.Tensor] = None,
                  stream: Optional[torch.cuda.Stream] = None):
    """dQw = X^T.dQ (fp32), dKw = X^T.dK, dVw = X^T.dV (bf16) over all B*M rows
    (attention.metal:344-393)."""
    act = (B, p.M, p.N)
    _check(x, "x", torch.bfloat16, act)
    _check(dQ, "dQ", torch.float32, act)
    _check(dK, "dK", torch.bfloat16, act)
    _check(dV, "dV", torch.bfloat16, act)
    w = (p.N, p.N)
    dQw = _out(dQw, x, w, torch.float32, "dQw")
    dKw = _out(dKw, x, w, torch.bfloat16, "dKw")
    dVw = _out(dVw, x, w, torch.bfloat16, "dVw")
    _lib.call("ma_computeGradDw", _ptr(x), _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(dQw), _ptr(dKw),
              _ptr(dVw), ctypes.byref(p), B, _stream(stream))
    return dQw, dKw, dVw


def flashAttentionForward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, p: AttentionParams,
                          B: int, out: Optional[torch.Tensor] = None,
                          l: Optional[torch.Tensor] = None, shard: Optional[tuple] = None,
                          stream: Optional[torch.cuda.Stream] = None):
    """out, l = causal attention of (q, k, v) (attention.metal:56-164).

    ``shard=(bh_begin, bh_end)`` restricts the work to flat (batch, head) indices
    in that range (ma_flashAttentionForward_shard)."""
    act = (B, p.M, p.N)
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check(t, n, torch.bfloat16, act)
    out = _out(out, q, act, torch.bfloat16, "out")
    l = _out(l, q, (B, p.M, p.NH), torch.float32, "l")
    if shard is None:
        _lib.call("ma_flashAttentionForward", _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(l),
                  ctypes.byref(p), B, _stream(stream))
    else:
        _lib.call("ma_flashAttentionForward_shard", _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(l),
                  ctypes.byref(p), B, shard[0], shard[1], _stream(stream))
    return out, l


def flashAttentionForwardComputeD(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dO: torch.Tensor,
                                  p: AttentionParams, B: int, out: Optional[torch.Tensor] = None,
                                  l: Optional[torch.Tensor] = None, D: Optional[torch.Tensor] = None,
                                  shard: Optional[tuple] = None, stream: Optional[torch.cuda.Stream] = None,
                                  zero_dQ: Optional[torch.Tensor] = None):
    """out, l, D = flashAttentionForward then computeD(dO, out), for callers
    that know dO before the forward (ma_flashAttentionForwardComputeD; at
    head size 64 D is formed in the forward's epilogue).  With zero_dQ (fp32
    [B, T, N]) the forward also writes zeros to it for every (row, head) it
    computes (ma_flashAttentionForwardComputeDZeroDQ), for a following
    flashAttentionBackward(..., accumulate_dQ=True)."""
    act = (B, p.M, p.N)
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (dO, "dO")):
        _check(t, n, torch.bfloat16, act)
    out = _out(out, q, act, torch.bfloat16, "out")
    l = _out(l, q, (B, p.M, p.NH), torch.float32, "l")
    D = _out(D, q, (B, p.M, p.NH), torch.bfloat16, "D")
    if zero_dQ is not None:
        _check(zero_dQ, "zero_dQ", torch.float32, act)
        name = "ma_flashAttentionForwardComputeDZeroDQ"
        args = (_ptr(q), _ptr(k), _ptr(v), _ptr(dO), _ptr(out), _ptr(l), _ptr(D), _ptr(zero_dQ),
                ctypes.byref(p), B)
        if shard is None:
            _lib.call(name, *args, _stream(stream))
        else:
            _lib.call(name + "_shard", *args, shard[0], shard[1], _stream(stream))
    elif shard is None:
        _lib.call("ma_flashAttentionForwardComputeD", _ptr(q), _ptr(k), _ptr(v), _ptr(dO), _ptr(out), _ptr(l),
                  _ptr(D), ctypes.byref(p), B, _stream(stream))
    else:
        _lib.call("ma_flashAttentionForwardComputeD_shard", _ptr(q), _ptr(k), _ptr(v), _ptr(dO), _ptr(out),
                  _ptr(l), _ptr(D), ctypes.byref(p), B, shard[0], shard[1], _stream(stream))
    return out, l, D


def computeD(dO: torch.Tensor, O: torch.Tensor, p: AttentionParams, B: int,
             D: Optional[torch.Tensor] = None, shard: Optional[tuple] = None,
             stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """D = rowsum(dO * O) per head, bf16 (attention.metal:166-195)."""
    act = (B, p.M, p.N)
    _check(dO, "dO", torch.bfloat16, act)
    _check(O, "O", torch.bfloat16, act)
    D = _out(D, dO, (B, p.M, p.NH), torch.bfloat16, "D")
    if shard is None:
        _lib.call("ma_computeD", _ptr(dO), _ptr(O), _ptr(D), ctypes.byref(p), B, _stream(stream))
    else:
        _lib.call("ma_computeD_shard", _ptr(dO), _ptr(O), _ptr(D), ctypes.byref(p), B, shard[0],
                  shard[1], _stream(stream))
    return D


def flashAttentionBackward(dZ: torch.Tensor, d: torch.Tensor, l: torch.Tensor, q: torch.Tensor,
                           k: torch.Tensor, v: torch.Tensor, p: AttentionParams, B: int,
                           dQ: Optional[torch.Tensor] = None, dK: Optional[torch.Tensor] = None,
                           dV: Optional[torch.Tensor] = None, shard: Optional[tuple] = None,
                           stream: Optional[torch.cuda.Stream] = None, accumulate_dQ: bool = False):
    """dQ (fp32), dK, dV (bf16) of causal attention (attention.metal:198-299).
    With accumulate_dQ, dQ (given) is added to, as the reference's kernel
    adds into a dQ its host zeroed (ma_flashAttentionBackwardAccumulate);
    otherwise dQ is written."""
    act = (B, p.M, p.N)
    for t, n in ((dZ, "dZ"), (q, "q"), (k, "k"), (v, "v")):
        _check(t, n, torch.bfloat16, act)
    _check(d, "d", torch.bfloat16, (B, p.M, p.NH))
    _check(l, "l", torch.float32, (B, p.M, p.NH))
    if accumulate_dQ and dQ is None:
        raise ValueError("accumulate_dQ needs the dQ tensor to add into")
    dQ = _out(dQ, q, act, torch.float32, "dQ")
    dK = _out(dK, q, act, torch.bfloat16, "dK")
    dV = _out(dV, q, act, torch.bfloat16, "dV")
    args = (_ptr(dZ), _ptr(d), _ptr(l), _ptr(q), _ptr(k), _ptr(v), _ptr(dQ), _ptr(dK), _ptr(dV),
            ctypes.byref(p), B)
    name = "ma_flashAttentionBackwardAccumulate" if accumulate_dQ else "ma_flashAttentionBackward"
    if shard is None:
        _lib.call(name, *args, _stream(stream))
    else:
        _lib.call(name + "_shard", *args, shard[0], shard[1], _stream(stream))
    return dQ, dK, dV


def device_status(stream: Optional[torch.cuda.Stream] = None) -> int:
    """Reads and clears the device's kernel status (0 = no bounded wait ran
    out; else a mask of the _lib.STATUS_* bits), for every entry point
    including flashAttentionBackward_noalloc."""
    st = ctypes.c_uint32(0)
    _lib.call("ma_device_status", ctypes.byref(st), _stream(stream))
    return st.value


def debug_expire_next_wait(kernels: int, wait_ns: int = 1_000_000) -> None:
    """Test hook of the time-out path: the next launch of each kernel in
    `kernels` (_lib.STATUS_FWD_TIMEOUT / _lib.STATUS_BWD_TIMEOUT) lets a wait
    run out after `wait_ns` and winds down as after a real time-out (its bit
    then shows in device_status).  kernels=0 cancels a pending request."""
    _lib.call("ma_debug_expire_next_wait", int(kernels), int(wait_ns))


class CudaAttention:
    """Attention core of one transformer block with reference-style buffers.

    Mirrors the attention part of the reference's MetalAttention harness
    (main.cpp:955-1284) and Model::forward/backward (model.h:446-473,
    639-665): buffers are allocated once for (B, T, NH, D) and reused, forward
    runs flashAttentionForward, backward runs computeD then
    flashAttentionBackward.  The projections around attention are not part of
    this path."""

    def __init__(self, B: int, T: int, NH: int, D: int, device="cuda"):
        self.B, self.T, self.NH, self.D = B, T, NH, D
        self.p = make_params(T, NH, D)
        act = (B, T, NH * D)
        dev = torch.device(device)
        self.out = torch.empty(act, dtype=torch.bfloat16, device=dev)
        self.l = torch.empty((B, T, NH), dtype=torch.float32, device=dev)
        self.Dvec = torch.empty((B, T, NH), dtype=torch.bfloat16, device=dev)
        self.dQ = torch.empty(act, dtype=torch.float32, device=dev)
        self.dK = torch.empty(act, dtype=torch.bfloat16, device=dev)
        self.dV = torch.empty(act, dtype=torch.bfloat16, device=dev)

    def forward(self, q, k, v, stream=None):
        self.q, self.k, self.v = q, k, v
        return flashAttentionForward(q, k, v, self.p, self.B, out=self.out, l=self.l,
                                     stream=stream)

    def backward(self, dO, stream=None):
        computeD(dO, self.out, self.p, self.B, D=self.Dvec, stream=stream)
        return flashAttentionBackward(dO, self.Dvec, self.l, self.q, self.k, self.v, self.p,
                                      self.B, dQ=self.dQ, dK=self.dK, dV=self.dV, stream=stream)


def _check_host(t: torch.Tensor, name: str, dtype: torch.dtype, shape: tuple) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.is_cuda:
        raise ValueError(f"{name} must be a host (CPU) tensor; use the device entry points for CUDA tensors")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.numel() != _numel(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class HostPipeline:
    """Attention over host-resident batches (ma_host_pipeline_*): the batch is
    split into chunks of `chunk_B` sequences whose host->device copies,
    kernels and device->host copies overlap on three internal streams.  The
    reference needs no such step (its Metal buffers are shared CPU/GPU memory,
    model.h:236-253); O, l, dK and dV equal the device entry points bit for
    bit, and dQ to fp32 rounding (its reduce-adds arrive in no fixed order).
    Host tensors should be pinned (`tensor.pin_memory()`) for the overlap."""

    def __init__(self, T: int, NH: int, D: int, chunk_B: int, device=None):
        self.p = make_params(T, NH, D)
        self.T, self.NH, self.D, self.chunk_B = T, NH, D, chunk_B
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("ma_host_pipeline_create", ctypes.byref(self.p), chunk_B, ctypes.byref(h))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.call("ma_host_pipeline_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _shapes(self, B: int):
        act = (B, self.T, self.NH * self.D)
        return act, (B, self.T, self.NH)

    def forward(self, q, k, v, B: int, out=None, l=None, stream=None):
        """flashAttentionForward of B host sequences -> (out bf16, l fp32), host."""
        act, rows = self._shapes(B)
        for t, n in ((q, "q"), (k, "k"), (v, "v")):
            _check_host(t, n, torch.bfloat16, act)
        out = torch.empty(act, dtype=torch.bfloat16).pin_memory() if out is None else out
        l = torch.empty(rows, dtype=torch.float32).pin_memory() if l is None else l
        _check_host(out, "out", torch.bfloat16, act)
        _check_host(l, "l", torch.float32, rows)
        with torch.cuda.device(self.device):
            _lib.call("ma_flashAttentionForward_host", self._h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      out.data_ptr(), l.data_ptr(), B, _stream(stream))
        return out, l

    def forward_backward(self, q, k, v, dO, B: int, out=None, l=None, dQ=None, dK=None, dV=None,
                         stream=None):
        """forward + computeD + backward of B host sequences ->
        (out, l, dQ, dK, dV), host tensors, ready when `stream` is."""
        act, rows = self._shapes(B)
        for t, n in ((q, "q"), (k, "k"), (v, "v"), (dO, "dO")):
            _check_host(t, n, torch.bfloat16, act)
        mk = lambda t, shape, dt: torch.empty(shape, dtype=dt).pin_memory() if t is None else t
        out, l = mk(out, act, torch.bfloat16), mk(l, rows, torch.float32)
        dQ, dK, dV = mk(dQ, act, torch.float32), mk(dK, act, torch.bfloat16), mk(dV, act, torch.bfloat16)
        for t, n, dt, shp in ((out, "out", torch.bfloat16, act), (l, "l", torch.float32, rows),
                              (dQ, "dQ", torch.float32, act), (dK, "dK", torch.bfloat16, act),
                              (dV, "dV", torch.bfloat16, act)):
            _check_host(t, n, dt, shp)
        with torch.cuda.device(self.device):
            _lib.call("ma_attentionForwardBackward_host", self._h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      dO.data_ptr(), out.data_ptr(), l.data_ptr(), dQ.data_ptr(), dK.data_ptr(),
                      dV.data_ptr(), B, _stream(stream))
        return out, l, dQ, dK, dV
