"""ma_flashAttentionBackward_noalloc: the backward pass for callers that cannot
let a library allocate device memory (their own arena owns the GPU's memory,
they run under a fixed memory budget, or they must not take the device
synchronisation of cudaMalloc/cudaFree).  Its D values and status word live in
a scratch array compiled into the library instead of a caller- or
library-allocated buffer.

Checked through the C ABI against the allocating entry points
(ma_computeD + ma_flashAttentionBackward) on two calls in a row with different
shapes and inputs, so that a second call which read the first call's scratch
would show; tolerance as in the other GPU parity tests (max-abs 2e-2,
relative-L2 1e-2).  Its kernels' time-out bit goes to a status word in the
same scratch, which ma_device_status (allocating nothing) reads and clears:
after the two calls it must read 0, and a wait made to run out through the
time-out test hook must show there.  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

from metalllm_b200 import _lib
from metalllm_b200.inputs import normal_bf16

MAX_ABS, REL_L2 = 2e-2, 1e-2
MAX_ENTRIES = 1 << 21   # MA_NOALLOC_MAX_D_ENTRIES in include/metalattn.h


def _params(T, H, D):
    return _lib.AttentionParams(T, H * D, D, H)


def test_noalloc_rejects_sizes_beyond_the_scratch(cuda_lib):
    """B*M*NH above the scratch maximum fails with MA_ERR_LIMIT and a message
    naming the limit, before any device work (no GPU needed)."""
    T, H, D = 4096, 16, 64
    B = MAX_ENTRIES // (T * H) + 1
    fake = ctypes.c_void_p(1 << 20)
    p = _params(T, H, D)
    rc = cuda_lib.ma_flashAttentionBackward_noalloc(*([fake] * 9), ctypes.byref(p), B, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_LIMIT"
    assert b"scratch maximum" in cuda_lib.ma_last_error_string()


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_points_on_two_calls():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import attention as A
    from oracle.oracle import compare

    lib = _lib.load()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())

    def up(bits, shape):
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).reshape(shape).cuda()

    cases = [(2, 512, 4, 64, 11), (1, 768, 2, 128, 12)]
    prepared = []
    for B, T, H, D, seed in cases:
        shape = (B, T, H * D)
        q, k, v, do = (up(normal_bf16(B * T * H * D, seed, s), shape) for s in (1, 2, 3, 4))
        prm = A.make_params(T, H, D)
        out, l = A.flashAttentionForward(q, k, v, prm, B)
        prepared.append((B, T, H, D, q, k, v, do, out, l))
    torch.cuda.synchronize()

    # two calls in a row of the allocation-free entry point
    got = []
    for B, T, H, D, q, k, v, do, out, l in prepared:
        dQ = torch.full(q.shape, float("nan"), dtype=torch.float32, device=q.device)
        dK = torch.full_like(q, float("nan"))
        dV = torch.full_like(q, float("nan"))
        p = _params(T, H, D)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _lib.call("ma_flashAttentionBackward_noalloc", ptr(do), ptr(out), ptr(l), ptr(q), ptr(k),
                  ptr(v), ptr(dQ), ptr(dK), ptr(dV), ctypes.byref(p), B, stream)
        got.append((dQ, dK, dV))
    torch.cuda.synchronize()

    # the allocating entry points on the same inputs
    for (B, T, H, D, q, k, v, do, out, l), (dQ, dK, dV) in zip(prepared, got):
        prm = A.make_params(T, H, D)
        Dv = A.computeD(do, out, prm, B)
        rQ, rK, rV = A.flashAttentionBackward(do, Dv, l, q, k, v, prm, B)
        torch.cuda.synchronize()
        for name, a, b in (("dQ", dQ, rQ), ("dK", dK, rK), ("dV", dV, rV)):
            a32 = a.float().cpu().numpy()
            b32 = b.float().cpu().numpy()
            assert np.isfinite(a32).all(), f"{name} (B={B} T={T} D={D}) not fully written"
            ok, mae, rl2 = compare(a32, b32, MAX_ABS, REL_L2)
            assert ok, f"{name} (B={B} T={T} D={D}): max_abs={mae:.3e} rel_l2={rl2:.3e}"
    # ma_device_status also reads (and clears) the scratch's status word
    assert A.device_status() == 0

    # a backward whose bounded wait runs out (time-out test hook) is reported
    # through the scratch's status word, and the next call is unaffected
    B, T, H, D, q, k, v, do, out, l = prepared[0]
    p = _params(T, H, D)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dQ, dK, dV = (torch.empty(q.shape, dtype=torch.float32, device=q.device), torch.empty_like(q),
                  torch.empty_like(q))
    A.debug_expire_next_wait(_lib.STATUS_BWD_TIMEOUT, 1_000_000)
    _lib.call("ma_flashAttentionBackward_noalloc", ptr(do), ptr(out), ptr(l), ptr(q), ptr(k),
              ptr(v), ptr(dQ), ptr(dK), ptr(dV), ctypes.byref(p), B, stream)
    assert A.device_status() == _lib.STATUS_BWD_TIMEOUT
    _lib.call("ma_flashAttentionBackward_noalloc", ptr(do), ptr(out), ptr(l), ptr(q), ptr(k),
              ptr(v), ptr(dQ), ptr(dK), ptr(dV), ctypes.byref(p), B, stream)
    torch.cuda.synchronize()
    for a, b in ((dQ, got[0][0]), (dK, got[0][1]), (dV, got[0][2])):
        ok, mae, rl2 = compare(a.float().cpu().numpy(), b.float().cpu().numpy(), 1e-5, 1e-6)
        assert ok, f"after the time-out: max_abs={mae:.3e} rel_l2={rl2:.3e}"
    assert A.device_status() == 0

    # a size beyond the scratch is refused on a GPU too, and changes nothing
    T, H, D = 4096, 16, 64
    B = MAX_ENTRIES // (T * H) + 1
    p = _params(T, H, D)
    q = prepared[0][4]
    rc = lib.ma_flashAttentionBackward_noalloc(*([ptr(q)] * 9), ctypes.byref(p), B, None)
    assert _lib.ERROR_NAMES[rc] == "MA_ERR_LIMIT"
