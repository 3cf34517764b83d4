"""Host side of the training step (config 5): a thin wrapper over the
ma_model_* C ABI (include/metalattn.h), the CUDA counterpart of the
reference's Model (model.h).  The model lives on the current CUDA device and
owns its buffers; forward/backward/step enqueue work on a torch CUDA stream.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib


class MaModelConfig(ctypes.Structure):
    _fields_ = [("B", ctypes.c_uint32), ("T", ctypes.c_uint32), ("E", ctypes.c_uint32),
                ("NH", ctypes.c_uint32), ("layers", ctypes.c_uint32), ("mlp_scale", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("lr", ctypes.c_float), ("seed", ctypes.c_uint64)]


_P = ctypes.c_void_p
_bound = False


def _bind():
    global _bound
    lib = _lib.load()
    if _bound:
        return lib
    sig = {
        "ma_model_create": ([ctypes.POINTER(MaModelConfig), ctypes.POINTER(_P)], ctypes.c_int),
        "ma_model_destroy": ([_P], ctypes.c_int),
        "ma_model_forward": ([_P, _P, _P, _P], ctypes.c_int),
        "ma_model_backward": ([_P, _P], ctypes.c_int),
        "ma_model_step": ([_P, _P], ctypes.c_int),
        "ma_model_tensor": ([_P, ctypes.c_char_p, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_uint64)],
                            ctypes.c_int),
        "ma_model_read": ([_P, ctypes.c_char_p, _P, ctypes.c_uint64], ctypes.c_int),
        "ma_model_write": ([_P, ctypes.c_char_p, _P, ctypes.c_uint64], ctypes.c_int),
        "ma_model_param_count": ([_P], ctypes.c_uint32),
        "ma_model_param_name": ([_P, ctypes.c_uint32], ctypes.c_char_p),
        "ma_model_status": ([_P, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
        "ma_model_last_error": ([], ctypes.c_char_p),
    }
    for n, (a, r) in sig.items():
        f = getattr(lib, n)
        f.argtypes = a
        f.restype = r
    _bound = True
    return lib


def _check(rc, what):
    if rc != 0:
        msg = _bind().ma_model_last_error().decode(errors="replace")
        raise _lib.MetalAttnError(rc, msg, what)


# gradients kept in fp32 (the reference's float atomic accumulators and dQw)
def _grad_is_f32(name: str) -> bool:
    """Gradients are fp32 except the positional embedding's (bf16, as the
    reference's dStream batch sum writes it); Adam rounds them to bf16."""
    return name != "pos"


class TrainingModel:
    """model.h's Model on CUDA for B sequences of length T (config 5:
    B=64, T=256, E=384, NH=6, layers=6, mlp_scale=2, vocab=128)."""

    def __init__(self, B=64, T=256, E=384, NH=6, layers=6, mlp_scale=2, vocab=128, lr=0.003, seed=0):
        lib = _bind()
        self.cfg = MaModelConfig(B, T, E, NH, layers, mlp_scale, vocab, lr, seed)
        h = _P()
        _check(lib.ma_model_create(ctypes.byref(self.cfg), ctypes.byref(h)), "ma_model_create")
        self._h = h
        self._tokens = self._targets = None

    def close(self):
        if self._h:
            _bind().ma_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _stream(stream: Optional[torch.cuda.Stream]):
        s = stream if stream is not None else torch.cuda.current_stream()
        return _P(s.cuda_stream)

    def forward(self, tokens: torch.Tensor, targets: torch.Tensor, stream=None):
        for t, n in ((tokens, "tokens"), (targets, "targets")):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous() or \
                    t.numel() != self.cfg.B * self.cfg.T:
                raise ValueError(f"{n} must be a contiguous int32 CUDA tensor of B*T elements")
            if t.device.index != torch.cuda.current_device():
                raise ValueError(f"{n} is on {t.device}, not on the current CUDA device")
        self._tokens, self._targets = tokens, targets  # kept alive until backward
        _check(_bind().ma_model_forward(self._h, _P(tokens.data_ptr()), _P(targets.data_ptr()),
                                        self._stream(stream)), "ma_model_forward")

    def backward(self, stream=None):
        _check(_bind().ma_model_backward(self._h, self._stream(stream)), "ma_model_backward")

    def step(self, stream=None):
        _check(_bind().ma_model_step(self._h, self._stream(stream)), "ma_model_step")

    def train_step(self, tokens, targets, stream=None):
        self.forward(tokens, targets, stream)
        self.backward(stream)
        self.step(stream)

    def param_names(self):
        lib = _bind()
        return [lib.ma_model_param_name(self._h, i).decode()
                for i in range(lib.ma_model_param_count(self._h))]

    def tensor_bytes(self, name: str) -> int:
        p, n = _P(), ctypes.c_uint64()
        _check(_bind().ma_model_tensor(self._h, name.encode(), ctypes.byref(p), ctypes.byref(n)), name)
        return n.value

    def read(self, name: str) -> np.ndarray:
        """Synchronous copy of a named tensor: bf16 as uint16 bits, fp32 as float32."""
        nbytes = self.tensor_bytes(name)
        if name.startswith("grad."):
            dt = np.float32 if _grad_is_f32(name[5:]) else np.uint16
        elif name in ("loss", "loss_rows", "lse_rows", "master"):
            dt = np.float32
        elif name.endswith(".mask"):
            dt = np.uint8
        else:
            dt = np.uint16
        out = np.empty(nbytes // np.dtype(dt).itemsize, dt)
        torch.cuda.synchronize()
        _check(_bind().ma_model_read(self._h, name.encode(), _P(out.ctypes.data), nbytes), name)
        return out

    def write(self, name: str, bits: np.ndarray):
        a = np.ascontiguousarray(bits)
        torch.cuda.synchronize()
        _check(_bind().ma_model_write(self._h, name.encode(), _P(a.ctypes.data), a.nbytes), name)

    def loss(self) -> float:
        return float(self.read("loss")[0])

    def status(self) -> int:
        s = ctypes.c_uint32()
        torch.cuda.synchronize()
        _check(_bind().ma_model_status(self._h, ctypes.byref(s)), "ma_model_status")
        return s.value
