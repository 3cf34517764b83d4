"""Host-resident batches through ma_host_pipeline_*: the chunked copy /
compute / copy-back pipeline gives the same bits as the device entry points
(forward with computeD, then backward) for O, l, dK and dV, and dQ to fp32
rounding (its bulk reduce-adds from different key tiles arrive in no fixed
order), since every (batch, head) is independent and chunking the batch
changes nothing; for a ragged last chunk, both head sizes, pinned and
pageable host memory, and repeated calls on one pipeline."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from metalllm_b200.inputs import normal_bf16  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def A():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import attention
    return attention


def _host(B, T, H, D, seed, pin):
    n = B * T * H * D
    ts = [torch.from_numpy(normal_bf16(n, seed, s, 1.0).view(np.int16)).view(torch.bfloat16).reshape(B, T, H * D)
          for s in range(4)]
    return [t.pin_memory() if pin else t for t in ts]


def _same(name, g, r):
    if name == "dQ":
        ref = r.double()
        assert (g.double() - ref).abs().max().item() <= 1e-5 * max(1.0, ref.abs().max().item()), name
    else:
        assert torch.equal(g, r), name


def _device_reference(A, q, k, v, dO, B, T, H, D):
    p = A.make_params(T, H, D)
    dq, dk, dv, ddo = (t.cuda() for t in (q, k, v, dO))
    out, l, Dv = A.flashAttentionForwardComputeD(dq, dk, dv, ddo, p, B)
    dQ, dK, dV = A.flashAttentionBackward(ddo, Dv, l, dq, dk, dv, p, B)
    torch.cuda.synchronize()
    return [t.cpu() for t in (out, l, dQ, dK, dV)]


@pytest.mark.parametrize("B,T,H,D,chunk,pin", [(5, 200, 3, 64, 2, True), (3, 256, 2, 128, 1, True),
                                               (4, 130, 2, 64, 4, False), (7, 1024, 2, 64, 3, True)])
def test_host_pipeline_matches_device_entry_points(A, B, T, H, D, chunk, pin):
    q, k, v, dO = _host(B, T, H, D, 71, pin)
    ref = _device_reference(A, q, k, v, dO, B, T, H, D)
    pl = A.HostPipeline(T, H, D, chunk)
    stream = torch.cuda.Stream()
    for _ in range(2):  # the second call reuses the slots and events
        got = pl.forward_backward(q, k, v, dO, B, stream=stream)
        stream.synchronize()
        assert A.device_status() == 0
        for name, g, r in zip(("out", "l", "dQ", "dK", "dV"), got, ref):
            _same(name, g, r)
    out, l = pl.forward(q, k, v, B, stream=stream)
    stream.synchronize()
    assert torch.equal(out, ref[0]) and torch.equal(l, ref[1])
    pl.close()


def test_host_pipeline_smaller_batch_than_chunk_and_errors(A):
    B, T, H, D = 2, 128, 2, 64
    q, k, v, dO = _host(B, T, H, D, 73, True)
    ref = _device_reference(A, q, k, v, dO, B, T, H, D)
    pl = A.HostPipeline(T, H, D, 8)
    got = pl.forward_backward(q, k, v, dO, B)
    torch.cuda.synchronize()
    for name, g, r in zip(("out", "l", "dQ", "dK", "dV"), got, ref):
        _same(name, g, r)
    with pytest.raises(ValueError):
        pl.forward(q.cuda(), k, v, B)
    with pytest.raises(A.MetalAttnError, match="MA_ERR_SHAPE"):
        A.HostPipeline(T, H, 32, 1)
    pl.close()
