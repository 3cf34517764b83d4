"""ctypes binding of libmetalattn.so (the C ABI declared in include/metalattn.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmetalattn.so"

MA_OK = 0
# bits of the status word read by ma_device_status (MA_STATUS_* in metalattn.h)
STATUS_FWD_TIMEOUT = 1 << 0
STATUS_BWD_TIMEOUT = 1 << 1
STATUS_QKV_TIMEOUT = 1 << 2
STATUS_GEMM_TIMEOUT = 1 << 3
ERROR_NAMES = {
    1: "MA_ERR_SHAPE",
    2: "MA_ERR_NULL",
    3: "MA_ERR_ALIGN",
    4: "MA_ERR_CUDA",
    5: "MA_ERR_DEVICE_TIMEOUT",
    6: "MA_ERR_RANGE",
    7: "MA_ERR_NO_DEVICE",
    8: "MA_ERR_LIMIT",
}


class AttentionParams(ctypes.Structure):
    """Mirror of the reference's AttentionParams (attention.metal:7-12)."""

    _fields_ = [("M", ctypes.c_uint32), ("N", ctypes.c_uint32),
                ("D", ctypes.c_uint32), ("NH", ctypes.c_uint32)]


class MetalAttnError(RuntimeError):
    def __init__(self, code: int, message: str, entry: str):
        self.code = code
        self.entry = entry
        super().__init__(f"{entry} failed with {ERROR_NAMES.get(code, code)}: {message}")


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_PP = ctypes.POINTER(AttentionParams)

# name -> argtypes (every entry returns int)
SIGNATURES = {
    "ma_computeQKV": [_P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionForward": [_P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_computeD": [_P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionForwardComputeD": [_P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionForwardComputeD_shard": [_P, _P, _P, _P, _P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_flashAttentionBackward": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionBackwardAccumulate": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionBackwardAccumulate_shard": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_flashAttentionForwardComputeDZeroDQ": [_P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_flashAttentionForwardComputeDZeroDQ_shard": [_P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_flashAttentionForward_shard": [_P, _P, _P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_computeD_shard": [_P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_flashAttentionBackward_shard": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _U32, _U32, _P],
    "ma_flashAttentionBackward_noalloc": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_projForward": [_P, _P, _P, _PP, _U32, _P],
    "ma_projBackwarddW": [_P, _P, _P, _PP, _U32, _P],
    "ma_projBackwarddX": [_P, _P, _P, _PP, _U32, _P],
    "ma_projBackwarddXComputeD": [_P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_computeGradDx": [_P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_computeGradDw": [_P, _P, _P, _P, _P, _P, _P, _PP, _U32, _P],
    "ma_host_pipeline_create": [_PP, _U32, ctypes.POINTER(_P)],
    "ma_host_pipeline_destroy": [_P],
    "ma_flashAttentionForward_host": [_P, _P, _P, _P, _P, _P, _U32, _P],
    "ma_attentionForwardBackward_host": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _P],
    "ma_device_status": [ctypes.POINTER(ctypes.c_uint32), _P],
    "ma_debug_expire_next_wait": [_U32, _U32],
    "ma_version": [],
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads libmetalattn.so (built in-tree by metalllm_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m metalllm_b200.build` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    lib.ma_kernel_launch_count.argtypes = []
    lib.ma_kernel_launch_count.restype = ctypes.c_uint64
    lib.ma_last_error_string.argtypes = []
    lib.ma_last_error_string.restype = ctypes.c_char_p
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Calls an entry point and raises MetalAttnError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != MA_OK:
        msg = lib.ma_last_error_string().decode(errors="replace")
        raise MetalAttnError(rc, msg, name)
