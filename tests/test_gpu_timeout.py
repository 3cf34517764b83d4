"""The time-out path of the kernels' bounded waits, on the GPU, without a fault.

The reference reports a failed command buffer and carries on
(model.h:358-366); here every mbarrier wait of the attention kernels is
bounded, and a wait that runs out makes the kernel wind down and set its bit
in the device status word.  ma_debug_expire_next_wait makes the next launch
of a kernel wait, with its first tensor-core products in flight, on an
mbarrier that nothing arrives at (a flag nothing sets) until a 1 ms limit
runs out.  Each test checks that the status reports exactly that kernel, and
that the next ordinary calls on the same device are bit-identical to the
calls before it (dQ to fp32 rounding: its key-tile partial sums arrive in no
fixed order), i.e. the wound-down launch freed its TMEM and left nothing
behind.  Nothing faults, traps or hangs: every wait, including the wind-down
waits for copies and products in flight, is bounded."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from metalllm_b200 import _lib  # noqa: E402
from metalllm_b200.inputs import normal_bf16  # noqa: E402

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000


@pytest.fixture(scope="module")
def A():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import attention
    yield attention
    attention.debug_expire_next_wait(0)


def _inputs(B, T, H, D, seed):
    shp = (B, T, H * D)
    return [torch.from_numpy(normal_bf16(B * T * H * D, seed, s).view(np.int16)).view(torch.bfloat16)
            .reshape(shp).cuda() for s in (1, 2, 3, 4)]


def _chain(A, q, k, v, do, p, B):
    out, l = A.flashAttentionForward(q, k, v, p, B)
    Dv = A.computeD(do, out, p, B)
    dQ, dK, dV = A.flashAttentionBackward(do, Dv, l, q, k, v, p, B)
    torch.cuda.synchronize()
    return out, l, Dv, dQ, dK, dV


def _same(a, b):
    for i in (0, 1, 2, 4, 5):
        assert torch.equal(a[i], b[i]), i
    assert torch.allclose(a[3], b[3], rtol=1e-5, atol=1e-5)


# (which kernel, head size, sequence length): the d=64 backward and forward
# of both schedules (static rounds up to 16 tiles, one CTA per unit under
# cluster launch control beyond, with a launch-control request in flight
# when the wait runs out), the d=128 backward (always launch control) and
# forward, and the forward with computeD fused at T=256, where the unit's
# diagonal tile is its first, so the dO tile load is in flight when the wait
# runs out
CASES = [("bwd", 64, 512), ("bwd", 64, 2304), ("bwd", 128, 512), ("fwd", 64, 512),
         ("fwd", 64, 2304), ("fwd", 128, 512), ("fwd_d", 64, 256)]


@pytest.mark.parametrize("kernel,D,T", CASES, ids=[f"{k}-d{d}-T{t}" for k, d, t in CASES])
def test_expired_wait_is_reported_and_the_device_recovers(A, kernel, D, T):
    B, H = 2, 3
    q, k, v, do = _inputs(B, T, H, D, seed=T + D)
    p = A.make_params(T, H, D)
    ref = _chain(A, q, k, v, do, p, B)
    assert A.device_status() == 0
    bit = _lib.STATUS_BWD_TIMEOUT if kernel == "bwd" else _lib.STATUS_FWD_TIMEOUT
    A.debug_expire_next_wait(bit, LIMIT_NS)
    if kernel == "bwd":
        A.flashAttentionBackward(do, ref[2], ref[1], q, k, v, p, B)
    elif kernel == "fwd":
        A.flashAttentionForward(q, k, v, p, B)
    else:
        A.flashAttentionForwardComputeD(q, k, v, do, p, B)
    torch.cuda.synchronize()
    assert A.device_status() == bit
    # the request was consumed by that launch: the next calls run normally
    again = _chain(A, q, k, v, do, p, B)
    _same(ref, again)
    assert A.device_status() == 0


def test_expire_request_is_validated(A):
    with pytest.raises(A.MetalAttnError, match="MA_ERR_RANGE"):
        A.debug_expire_next_wait(_lib.STATUS_QKV_TIMEOUT, LIMIT_NS)
    with pytest.raises(A.MetalAttnError, match="MA_ERR_RANGE"):
        A.debug_expire_next_wait(_lib.STATUS_FWD_TIMEOUT, 0)
    A.debug_expire_next_wait(_lib.STATUS_FWD_TIMEOUT, LIMIT_NS)
    A.debug_expire_next_wait(0)  # cancelled: the next forward runs normally
    B, T, H, D = 1, 256, 2, 64
    q, k, v, do = _inputs(B, T, H, D, seed=5)
    p = A.make_params(T, H, D)
    A.flashAttentionForward(q, k, v, p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
