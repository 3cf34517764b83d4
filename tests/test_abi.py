"""CPU tests of the C ABI: the library loads, exports every symbol that
include/metalattn.h declares, the header compiles as C and C++, and argument
validation rejects bad calls before any device work (no GPU needed)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "metalattn.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"MA_API\s+[\w\s\*]+?\b(ma_\w+)\s*\(", text)))


def test_header_declares_the_four_kernels():
    syms = declared_symbols()
    for name in ("ma_computeQKV", "ma_flashAttentionForward", "ma_computeD",
                 "ma_flashAttentionBackward"):
        assert name in syms


def test_library_exports_every_declared_symbol(cuda_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "metalllm_b200" / "libmetalattn.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ma_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    for s in declared_symbols():
        assert hasattr(cuda_lib, s)


@pytest.mark.parametrize("lang,compiler", [("c", "gcc"), ("c++", "g++")])
def test_header_compiles(tmp_path, lang, compiler):
    src = tmp_path / ("t.c" if lang == "c" else "t.cpp")
    src.write_text('#include "metalattn.h"\n'
                   '_Static_assert(sizeof(AttentionParams) == 16, "AttentionParams is 16 bytes");\n'
                   if lang == "c" else
                   '#include "metalattn.h"\n'
                   'static_assert(sizeof(AttentionParams) == 16, "AttentionParams is 16 bytes");\n'
                   'int main() { AttentionParams p{256, 384, 64, 6}; return ma_version() > 0 ? 0 : (int)p.M; }\n')
    cmd = [compiler, "-Wall", "-Werror", "-I", str(ROOT / "include"), "-c", str(src), "-o",
           str(tmp_path / "t.o")]
    subprocess.run(cmd, check=True)


def test_cpp_host_links_and_runs_version(tmp_path, cuda_lib):
    """A C++ host (as the reference's model.h would be) links against the
    library and calls an entry point that needs no device."""
    src = tmp_path / "host.cpp"
    src.write_text('#include "metalattn.h"\n#include <cstdio>\n'
                   'int main() { std::printf("%d\\n", ma_version()); return 0; }\n')
    exe = tmp_path / "host"
    libdir = ROOT / "metalllm_b200"
    subprocess.run(["g++", "-I", str(ROOT / "include"), str(src), "-L", str(libdir), "-lmetalattn",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    assert int(out.strip()) == cuda_lib.ma_version()


def _params(M=256, N=384, D=64, NH=6):
    from metalllm_b200._lib import AttentionParams
    return AttentionParams(M, N, D, NH)


def _err(lib):
    return lib.ma_last_error_string().decode()


ALIGNED = 1 << 20  # a fake (never dereferenced) 16-byte aligned address


@pytest.mark.parametrize("params,code", [
    (dict(D=32, N=192), 1),              # unsupported head size
    (dict(N=383), 1),                    # N != NH*D
    (dict(D=96, N=384), 1),              # head size 96
    (dict(NH=0, N=0), 1),                # empty
])
def test_forward_rejects_bad_shapes_without_device(cuda_lib, params, code):
    p = _params(**params)
    rc = cuda_lib.ma_flashAttentionForward(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                           ctypes.byref(p), 1, None)
    assert rc == code, _err(cuda_lib)
    assert _err(cuda_lib)


def test_null_and_misaligned_pointers_rejected(cuda_lib):
    p = _params()
    rc = cuda_lib.ma_flashAttentionForward(None, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ctypes.byref(p), 1, None)
    assert rc == 2 and "'q'" in _err(cuda_lib)
    rc = cuda_lib.ma_flashAttentionForward(ALIGNED, ALIGNED + 2, ALIGNED, ALIGNED, ALIGNED, ctypes.byref(p), 1, None)
    assert rc == 3 and "'k'" in _err(cuda_lib)
    rc = cuda_lib.ma_flashAttentionBackward(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, None,
                                            ALIGNED, ALIGNED, ctypes.byref(p), 1, None)
    assert rc == 2 and "'dQ'" in _err(cuda_lib)
    rc = cuda_lib.ma_computeD(ALIGNED, ALIGNED, ALIGNED + 1, ctypes.byref(p), 1, None)
    assert rc == 3
    rc = cuda_lib.ma_flashAttentionForward(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, None, 1, None)
    assert rc == 2


def test_shard_range_rejected(cuda_lib):
    p = _params()
    rc = cuda_lib.ma_flashAttentionForward_shard(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                                 ctypes.byref(p), 2, 0, 13, None)
    assert rc == 6, _err(cuda_lib)
    rc = cuda_lib.ma_flashAttentionBackward_shard(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                                  ALIGNED, ALIGNED, ALIGNED, ctypes.byref(p), 2, 5, 4, None)
    assert rc == 6
    rc = cuda_lib.ma_computeD_shard(ALIGNED, ALIGNED, ALIGNED, ctypes.byref(p), 2, 3, 99, None)
    assert rc == 6


def test_qkv_rejects_bad_shapes(cuda_lib):
    p = _params(N=100)
    rc = cuda_lib.ma_computeQKV(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                ctypes.byref(p), 1, None)
    assert rc == 1


def test_valid_call_without_gpu_fails_cleanly(cuda_lib):
    """On a machine without an sm_100 device a valid call returns an error code
    (no crash, no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = _params()
    rc = cuda_lib.ma_flashAttentionForward(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ctypes.byref(p), 1, None)
    assert rc in (4, 7), _err(cuda_lib)


def test_python_api_refuses_cpu_tensors():
    import torch
    from metalllm_b200 import attention as A
    p = A.make_params(64, 1, 64)
    x = torch.zeros(1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        A.flashAttentionForward(x, x, x, p, 1)


def test_forward_compute_d_validates_its_extra_buffers(cuda_lib):
    """ma_flashAttentionForwardComputeD checks dO and D like every other
    buffer, before any device work."""
    p = _params()
    rc = cuda_lib.ma_flashAttentionForwardComputeD(ALIGNED, ALIGNED, ALIGNED, None, ALIGNED, ALIGNED, ALIGNED,
                                                   ctypes.byref(p), 1, None)
    assert rc == 2 and "'dO'" in _err(cuda_lib)
    rc = cuda_lib.ma_flashAttentionForwardComputeD(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, None,
                                                   ctypes.byref(p), 1, None)
    assert rc == 2 and "'D'" in _err(cuda_lib)
    rc = cuda_lib.ma_flashAttentionForwardComputeD(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                                   ALIGNED + 1, ctypes.byref(p), 1, None)
    assert rc == 3 and "'D'" in _err(cuda_lib)
    bad = _params(N=383)
    rc = cuda_lib.ma_flashAttentionForwardComputeD(ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                                   ctypes.byref(bad), 1, None)
    assert rc == 1


def test_host_pipeline_validates_before_allocating(cuda_lib):
    """The host-buffer pipeline rejects bad shapes, a zero chunk and NULL
    outputs without touching a device; its run entry points reject a NULL
    pipeline, and destroying NULL is a no-op."""
    out = ctypes.c_void_p(ALIGNED)
    bad = _params(D=96, N=384)
    assert cuda_lib.ma_host_pipeline_create(ctypes.byref(bad), 8, ctypes.byref(out)) == 1
    assert out.value is None  # cleared on failure
    p = _params()
    assert cuda_lib.ma_host_pipeline_create(ctypes.byref(p), 0, ctypes.byref(out)) == 1
    assert cuda_lib.ma_host_pipeline_create(ctypes.byref(p), 8, None) == 2
    rc = cuda_lib.ma_flashAttentionForward_host(None, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, 8, None)
    assert rc == 2, _err(cuda_lib)
    rc = cuda_lib.ma_attentionForwardBackward_host(None, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED, ALIGNED,
                                                   ALIGNED, ALIGNED, ALIGNED, 8, None)
    assert rc == 2
    assert cuda_lib.ma_host_pipeline_destroy(None) == 0


def test_host_pipeline_without_gpu_fails_cleanly(cuda_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    out = ctypes.c_void_p()
    p = _params()
    rc = cuda_lib.ma_host_pipeline_create(ctypes.byref(p), 8, ctypes.byref(out))
    assert rc in (4, 7), _err(cuda_lib)
    assert out.value is None


def test_model_create_validates_its_configuration():
    """ma_model_create rejects empty, inconsistent and oversized
    configurations before it touches a device, and leaves *model NULL."""
    import torch
    from metalllm_b200 import train as T
    lib = T._bind()
    h = ctypes.c_void_p(ALIGNED)

    def create(**kw):
        c = dict(B=2, T=64, E=128, NH=2, layers=1, mlp_scale=2, vocab=128, lr=0.003, seed=0)
        c.update(kw)
        cfg = T.MaModelConfig(c["B"], c["T"], c["E"], c["NH"], c["layers"], c["mlp_scale"], c["vocab"], c["lr"],
                              c["seed"])
        return lib.ma_model_create(ctypes.byref(cfg), ctypes.byref(h))

    assert lib.ma_model_create(None, ctypes.byref(h)) == 2
    assert create(B=0) == 1 and h.value is None
    assert create(NH=3) == 1                # head size 128/3
    assert create(E=96, NH=1) == 1          # head size 96
    assert create(vocab=100) == 1           # vocabulary not a multiple of 64
    assert create(E=32768, NH=256) == 8     # E above 16384
    assert create(mlp_scale=1024) == 8      # MLP width above 65536
    assert create(vocab=1 << 21) == 8       # vocabulary above 2^20
    if not torch.cuda.is_available():
        assert create() in (4, 7), lib.ma_model_last_error()
        assert h.value is None


def test_expire_hook_validates_without_device(cuda_lib):
    """ma_debug_expire_next_wait (the time-out test hook) accepts only the
    kernels that have the hook and a wait of 1 ns .. 1 s; checked on the host."""
    from metalllm_b200 import _lib
    assert _lib.ERROR_NAMES[cuda_lib.ma_debug_expire_next_wait(_lib.STATUS_QKV_TIMEOUT, 1000)] == "MA_ERR_RANGE"
    assert _lib.ERROR_NAMES[cuda_lib.ma_debug_expire_next_wait(_lib.STATUS_BWD_TIMEOUT, 0)] == "MA_ERR_RANGE"
    assert _lib.ERROR_NAMES[cuda_lib.ma_debug_expire_next_wait(_lib.STATUS_BWD_TIMEOUT, 2 * 10 ** 9)] == "MA_ERR_RANGE"
    assert cuda_lib.ma_debug_expire_next_wait(_lib.STATUS_BWD_TIMEOUT, 1000) == 0
    assert cuda_lib.ma_debug_expire_next_wait(0, 0) == 0  # cancels the request


def test_zero_dq_and_accumulate_validate_without_device(cuda_lib):
    """The forward that zeroes dQ refuses a NULL or misaligned dQ, and the
    accumulating backward validates like ma_flashAttentionBackward, before
    any device work."""
    from metalllm_b200 import _lib
    p = _lib.AttentionParams(256, 128, 64, 2)
    fake = ctypes.c_void_p(1 << 20)
    odd = ctypes.c_void_p((1 << 20) + 4)
    rc = cuda_lib.ma_flashAttentionForwardComputeDZeroDQ(*([fake] * 7), None, ctypes.byref(p), 1, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_NULL" and b"'dQ'" in cuda_lib.ma_last_error_string()
    rc = cuda_lib.ma_flashAttentionForwardComputeDZeroDQ(*([fake] * 7), odd, ctypes.byref(p), 1, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_ALIGN"
    rc = cuda_lib.ma_flashAttentionBackwardAccumulate(*([fake] * 9), ctypes.byref(_lib.AttentionParams(256, 96, 32, 3)), 1, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_SHAPE"
    rc = cuda_lib.ma_flashAttentionBackwardAccumulate_shard(*([fake] * 9), ctypes.byref(p), 1, 0, 3, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_RANGE"
